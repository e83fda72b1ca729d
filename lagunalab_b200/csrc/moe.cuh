// Shared declarations for the MoE expert kernels.
#pragma once

#include "common.cuh"

namespace lg {

// Expert-parallel return of the down products (ep.cu): a routed pick p = row * k + j of a
// received row writes bf16(bf16(y) * w[p]) into the combine rows of the source rank that sent
// the row, ret[row / Tr] + (tok[row] * k + j) * H (peer memory), instead of a local buffer.
struct EpRet {
  __nv_bfloat16* ret[8];
  const int32_t* tok;
  const __nv_bfloat16* w;
  int Tr;
  int on;
};

__device__ __forceinline__ __nv_bfloat16* ep_ret_row(const EpRet& ep, int p, int k, int H,
                                                     float* wt) {
  const int row = p / k, j = p - row * k;
  *wt = __bfloat162float(ep.w[p]);
  return ep.ret[row / ep.Tr] + ((size_t)ep.tok[row] * k + j) * H;
}

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
  EpRet ep;                // expert-parallel return (ep.on), replacing ypick
  int* err;                // status word: a bounded wait that expired records a code here
  float* xg;               // [T, H/64] scratch (GEMV path): each token's 64-group sums of x
};

// The status word of the tensor-core workspace (lg_moe_status reads it); the GEMV kernels
// record their expired waits there too.
int* tc_err_word(void* tc_ws, int T, int H, int I, int I_sh, int E, int k);

// scratch: plan_scratch_bytes(T, k, E) bytes (null: the one-CTA-per-group kernel at any size)
int launch_plan(const int32_t* inds, int T, int k, int E, int with_shared, int32_t* counts,
                int32_t* offsets, int32_t* perm, int32_t* active, cudaStream_t s,
                int32_t* scratch);
size_t plan_scratch_bytes(int T, int k, int E);
int launch_gemv(const GemvArgs& a, int max_groups, cudaStream_t s);
// out[t] = bf16(bf16(bf16(sum_j bf16(y[t*k+j] * w[t*k+j])) * scale) + y[P + t]) per token, the
// picks summed in order j = 0..k-1 (picks whose expert id is outside [0, E) skipped), the shared
// row added when has_shared.
int moe_experts_ep(const void* x, int T, int H, int I, int E, int k, const int32_t* inds,
                   const void* weights, const uint32_t* const* q, const void* const* sc,
                   const void* const* bi, int path, void* workspace, size_t workspace_bytes,
                   const EpRet& ep, cudaStream_t st);
size_t moe_ep_workspace_bytes(int T, int H, int I, int E, int k);
int launch_combine(const __nv_bfloat16* yrows, const int32_t* inds, const __nv_bfloat16* w,
                   int T, int k, int E, int H, float routed_scale, int has_shared,
                   __nv_bfloat16* out, cudaStream_t s);

}  // namespace lg
