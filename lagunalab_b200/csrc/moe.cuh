// Shared declarations for the MoE expert kernels.
#pragma once

#include "common.cuh"

namespace lg {

// Arguments of the expert-product kernels.  Group g < E is routed expert g; group E (when
// present) is the shared expert.  Rows of group g are [offsets[g], offsets[g+1]) in the
// expert-contiguous order; perm[row] is the pick id (routed: t*k + j, shared: P + t).
struct GemvArgs {
  const __nv_bfloat16* x;  // [T, H]
  int T, H, I, I_sh, E, k, P;
  const int32_t* offsets;  // [E + 2]
  const int32_t* perm;     // [P + T]
  const int32_t* active;   // [1 + groups]: count, then group ids with rows
  const uint32_t *g_q, *u_q, *d_q;
  const __nv_bfloat16 *g_s, *g_b, *u_s, *u_b, *d_s, *d_b;
  const uint32_t *sg_q, *su_q, *sd_q;
  const __nv_bfloat16 *sg_s, *sg_b, *su_s, *su_b, *sd_s, *sd_b;
  __nv_bfloat16* h;        // [P + T, h_stride] intermediate (SwiGLU output), bf16
  int h_stride;
  __nv_bfloat16* ypick;    // [P (+ T with the shared expert), H] per-pick down outputs
};

int launch_plan(const int32_t* inds, int T, int k, int E, int with_shared, int32_t* counts,
                int32_t* offsets, int32_t* perm, int32_t* active, cudaStream_t s);
int launch_gemv(const GemvArgs& a, int max_groups, cudaStream_t s);
// out[t] = bf16(bf16(bf16(sum_j bf16(y[t*k+j] * w[t*k+j])) * scale) + y[P + t]) per token, the
// picks summed in order j = 0..k-1 (picks whose expert id is outside [0, E) skipped), the shared
// row added when has_shared.
int launch_combine(const __nv_bfloat16* yrows, const int32_t* inds, const __nv_bfloat16* w,
                   int T, int k, int E, int H, float routed_scale, int has_shared,
                   __nv_bfloat16* out, cudaStream_t s);

}  // namespace lg
