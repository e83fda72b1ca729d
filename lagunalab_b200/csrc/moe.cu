// MoE block orchestration: routing plan -> expert products -> combine, behind the C ABI.
//
// lg_moe_experts:  laguna_mlx/laguna.py:147-150 after route(); SwitchGLU per pick, then the
//                  weighted sum, routed scale and shared expert with the MLX graph's bf16
//                  rounding points, summed in a fixed order (deterministic).
// lg_switch_glu:   SwitchGLU(x, indices) per-pick outputs (mlx-lm switch_layers surface).
// lg_qmlp:         dense quantized SwiGLU MLP (laguna.py:114-122): the shared-expert machinery
//                  with no routed experts.
#include "moe.cuh"

namespace lg {

int launch_tc(const GemvArgs& a, int max_groups, void* tc_ws, cudaStream_t s);
size_t tc_workspace_bytes(int T, int H, int I, int I_sh, int E, int k);
bool tc_supported(int H, int I, int I_sh, int E);
int tc_status(const void* tc_ws, int T, int H, int I, int I_sh, int E, int k, int* status);

struct MoeWs {
  int32_t* counts;
  int32_t* offsets;
  int32_t* active;
  int32_t* perm;
  __nv_bfloat16* h;
  __nv_bfloat16* yrows;  // [P + T, H] per-pick down outputs (combine mode)
  void* tc;
  int32_t* plan;         // segmented-plan scratch (many picks)
  float* xg;             // [T, H/64] per-token group sums of x (GEMV path)
};

static size_t carve_moe(void* base, int T, int H, int I, int E, int k, int I_sh, MoeWs* w,
                        bool with_yrows = true) {
  Carver c(base);
  const int P = T * k;
  const int Imax = I > I_sh ? I : I_sh;
  MoeWs t;
  t.counts = c.take<int32_t>(E + 2);
  t.offsets = c.take<int32_t>(E + 2);
  t.active = c.take<int32_t>(E + 3);
  t.perm = c.take<int32_t>((size_t)P + T);
  t.h = c.take<__nv_bfloat16>(((size_t)P + T) * Imax);
  t.yrows = c.take<__nv_bfloat16>(with_yrows ? ((size_t)P + T) * H : 0);
  t.tc = c.take<char>(tc_workspace_bytes(T, H, I, I_sh, E, k));
  t.plan = c.take<int32_t>(plan_scratch_bytes(T, k, E) / sizeof(int32_t));
  t.xg = c.take<float>((size_t)T * (H / 64));
  if (w) *w = t;
  return align_up(c.used, 256);
}

__device__ __forceinline__ void bf16x8(uint4 v, float* f) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(u[j] << 16);
    f[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
  }
}

constexpr int CB_J = 8;  // picks whose rows a thread loads at once

// laguna.py:149-150 with the MLX graph's bf16 materialisation points: per pick
// bf16(y * w), their fp32 sum in pick order rounded to bf16, times the routed scale (bf16),
// plus the shared expert's row (bf16). One thread per 8 columns of a token; the order of
// every sum is fixed, so the result does not depend on scheduling.

__global__ void __launch_bounds__(256) combine_rows_kernel(const __nv_bfloat16* __restrict__ y,
                                    const int32_t* __restrict__ inds,
                                    const __nv_bfloat16* __restrict__ w, int T, int k, int E,
                                    int H, float scale, int has_shared,
                                    __nv_bfloat16* __restrict__ out) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  const int H8 = H / 8;
  const size_t total = (size_t)T * H8, P = (size_t)T * k;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / H8;
    const int c = (int)(i % H8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 shv = make_uint4(0u, 0u, 0u, 0u);
    if (has_shared) shv = *reinterpret_cast<const uint4*>(y + (P + t) * H + c);
    // up to CB_J picks at a time: their ids and weights, then all their row loads in flight
    // together, then the sum in pick order
    for (int j0 = 0; j0 < k; j0 += CB_J) {
      const int n = min(CB_J, k - j0);
      bool ok[CB_J];
      float wj[CB_J];
      uint4 rv[CB_J];
#pragma unroll
      for (int j = 0; j < CB_J; ++j) {
        ok[j] = false;
        wj[j] = 0.f;
        if (j < n) {
          const size_t p = t * k + j0 + j;
          const int e = inds[p];
          ok[j] = e >= 0 && e < E;
          wj[j] = bf2f(w[p]);
        }
      }
#pragma unroll
      for (int j = 0; j < CB_J; ++j)
        if (ok[j]) rv[j] = *reinterpret_cast<const uint4*>(y + (t * k + j0 + j) * H + c);
#pragma unroll
      for (int j = 0; j < CB_J; ++j) {
        if (!ok[j]) continue;
        float v[8];
        bf16x8(rv[j], v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += round_bf16(v[q] * wj[j]);
      }
    }
    float sh[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (has_shared) bf16x8(shv, sh);
    float r[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float s_ = round_bf16(round_bf16(acc[q]) * scale);
      r[q] = has_shared ? s_ + sh[q] : s_;
    }
    uint4 o;
    __nv_bfloat162 b0 = __floats2bfloat162_rn(r[0], r[1]), b1 = __floats2bfloat162_rn(r[2], r[3]);
    __nv_bfloat162 b2 = __floats2bfloat162_rn(r[4], r[5]), b3 = __floats2bfloat162_rn(r[6], r[7]);
    o.x = *reinterpret_cast<uint32_t*>(&b0);
    o.y = *reinterpret_cast<uint32_t*>(&b1);
    o.z = *reinterpret_cast<uint32_t*>(&b2);
    o.w = *reinterpret_cast<uint32_t*>(&b3);
    *reinterpret_cast<uint4*>(out + t * H + c) = o;
  }
}

int launch_combine(const __nv_bfloat16* yrows, const int32_t* inds, const __nv_bfloat16* w,
                   int T, int k, int E, int H, float routed_scale, int has_shared,
                   __nv_bfloat16* out, cudaStream_t st) {
  if (T <= 0) return LG_OK;
  const size_t n = (size_t)T * (H / 8);
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  prof_begin("combine", st);
  LG_CUDA_TRY(launch_k(combine_rows_kernel, dim3(blocks), dim3(256), 0, st, yrows, inds, w, T, k,
                       E, H, routed_scale, has_shared, out));
  prof_end("combine", st);
  LG_LAUNCH_CHECK("combine_rows");
  return LG_OK;
}

static int check_qmat(const void* q, const void* s, const void* b, const char* name) {
  if (!q || !s || !b) return fail(LG_ERR_INVALID, "%s: NULL weight/scales/biases", name);
  if (!aligned(q, 16) || !aligned(s, 2) || !aligned(b, 2))
    return fail(LG_ERR_INVALID, "%s: weight must be 16-byte aligned", name);
  return LG_OK;
}

// Common driver. mode: 0 = combine into bf16 out, 1 = per-pick SwitchGLU outputs.
static int moe_run(const void* x, int T, int H, int I, int E, int k, const int32_t* inds,
                   const void* weights, float routed_scale, const uint32_t* const* q,
                   const void* const* sc, const void* const* bi, int I_sh,
                   const uint32_t* const* sq, const void* const* ss, const void* const* sb,
                   int group_size, int bits, int path, void* out, void* workspace,
                   size_t workspace_bytes, int mode, cudaStream_t st,
                   const EpRet* ep = nullptr) {
  LG_CHECK_ARG(bits == 4 && group_size == 64,
               "experts: only 4-bit group-64 weights are supported (got bits=%d group=%d)", bits,
               group_size);
  LG_CHECK_ARG(T >= 0 && H > 0 && E >= 0 && E <= 256 && k >= 0 && I_sh >= 0,
               "experts: bad sizes T=%d H=%d E=%d k=%d", T, H, E, k);
  LG_CHECK_ARG(E == 0 || (k >= 1 && k <= E && I > 0), "experts: k=%d I=%d invalid for E=%d", k,
               I, E);
  LG_CHECK_ARG(H % 64 == 0 && (E == 0 || I % 64 == 0) && I_sh % 64 == 0,
               "experts: hidden %d and intermediate %d/%d must be multiples of 64", H, I, I_sh);
  LG_CHECK_ARG(path >= LG_PATH_AUTO && path <= LG_PATH_TENSOR, "experts: path %d", path);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(mode == 2 ? (ep != nullptr) : (out != nullptr && aligned(out, 16)),
               "experts: NULL or misaligned output");
  LG_CHECK_ARG(x && aligned(x, 16),
               "experts: x must be non-NULL and 16-byte aligned");
  if (E > 0) {
    LG_CHECK_ARG(inds != nullptr, "experts: NULL inds");
    LG_CHECK_ARG(mode == 1 || weights != nullptr, "experts: NULL routing weights");
    for (int j = 0; j < 3; ++j) {
      int rc = check_qmat(q[j], sc[j], bi[j], "experts");
      if (rc) return rc;
    }
  }
  if (I_sh > 0)
    for (int j = 0; j < 3; ++j) {
      int rc = check_qmat(sq[j], ss[j], sb[j], "shared expert");
      if (rc) return rc;
    }
  const int Ie = E > 0 ? I : 0;
  const size_t need = carve_moe(nullptr, T, H, Ie, E, k, I_sh, nullptr, mode == 0);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "experts: workspace %zu bytes at %p, need %zu (256-aligned)",
                workspace_bytes, workspace, need);
  if (T == 0) return LG_OK;
  MoeWs w;
  carve_moe(workspace, T, H, Ie, E, k, I_sh, &w, mode == 0);
  const int P = T * (E > 0 ? k : 0);
  const bool with_sh = I_sh > 0;
  if (mode == 1) LG_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(uint16_t) * (size_t)P * H, st));
  int rc = launch_plan(inds, T, E > 0 ? k : 0, E, with_sh ? 1 : 0, w.counts, w.offsets, w.perm,
                       w.active, st, w.plan);
  if (rc) return rc;
  GemvArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.T = T;
  a.H = H;
  a.I = Ie;
  a.I_sh = I_sh;
  a.E = E;
  a.k = E > 0 ? k : 0;
  a.P = P;
  a.offsets = w.offsets;
  a.perm = w.perm;
  a.active = w.active;
  a.g_q = q[0];
  a.u_q = q[1];
  a.d_q = q[2];
  a.g_s = static_cast<const __nv_bfloat16*>(sc[0]);
  a.u_s = static_cast<const __nv_bfloat16*>(sc[1]);
  a.d_s = static_cast<const __nv_bfloat16*>(sc[2]);
  a.g_b = static_cast<const __nv_bfloat16*>(bi[0]);
  a.u_b = static_cast<const __nv_bfloat16*>(bi[1]);
  a.d_b = static_cast<const __nv_bfloat16*>(bi[2]);
  a.sg_q = sq[0];
  a.su_q = sq[1];
  a.sd_q = sq[2];
  a.sg_s = static_cast<const __nv_bfloat16*>(ss[0]);
  a.su_s = static_cast<const __nv_bfloat16*>(ss[1]);
  a.sd_s = static_cast<const __nv_bfloat16*>(ss[2]);
  a.sg_b = static_cast<const __nv_bfloat16*>(sb[0]);
  a.su_b = static_cast<const __nv_bfloat16*>(sb[1]);
  a.sd_b = static_cast<const __nv_bfloat16*>(sb[2]);
  a.h = w.h;
  a.h_stride = Ie > I_sh ? Ie : I_sh;
  // combine mode: every pick row and shared row goes to the workspace, then one fixed-order
  // pass combines them; per-pick mode: the routed rows go straight to the caller's output
  a.ypick = mode == 0 ? w.yrows : static_cast<__nv_bfloat16*>(out);
  a.ep = {};
  if (mode == 2) a.ep = *ep;  // expert parallel: down outputs go to the source ranks
  a.err = tc_err_word(w.tc, T, H, Ie, I_sh, E, k);
  a.xg = w.xg;
  int max_groups = (E < P ? E : P) + (with_sh ? 1 : 0);
  // Tensor-core grouped GEMM when there are enough rows per expert to fill 128-row tiles;
  // the split-K GEMV otherwise (decode), or when the shapes do not tile.
  const bool tiles_ok = tc_supported(H, Ie, I_sh, E);
  const bool use_tc = (path == LG_PATH_TENSOR) ||
                      (path == LG_PATH_AUTO && tiles_ok && P + (with_sh ? T : 0) > LG_MOE_GEMV_MAX_ROWS);
  if (use_tc) {
    rc = launch_tc(a, max_groups, w.tc, st);  // clears the status word itself
  } else {
    LG_CUDA_TRY(cudaMemsetAsync(a.err, 0, sizeof(int), st));
    rc = launch_gemv(a, max_groups, st);
  }
  if (rc) return rc;
  if (mode == 0)
    return launch_combine(w.yrows, inds, static_cast<const __nv_bfloat16*>(weights), T, a.k, E, H,
                          routed_scale, with_sh ? 1 : 0, static_cast<__nv_bfloat16*>(out), st);
  return LG_OK;
}

// Expert products of received rows whose down outputs go back to their source ranks (ep.cu).
int moe_experts_ep(const void* x, int T, int H, int I, int E, int k, const int32_t* inds,
                   const void* weights, const uint32_t* const* q, const void* const* sc,
                   const void* const* bi, int path, void* workspace, size_t workspace_bytes,
                   const EpRet& ep, cudaStream_t st) {
  const uint32_t* nq[3] = {nullptr, nullptr, nullptr};
  const void* nv[3] = {nullptr, nullptr, nullptr};
  return moe_run(x, T, H, I, E, k, inds, weights, 1.0f, q, sc, bi, 0, nq, nv, nv, 64, 4, path,
                 nullptr, workspace, workspace_bytes, 2, st, &ep);
}

size_t moe_ep_workspace_bytes(int T, int H, int I, int E, int k) {
  return carve_moe(nullptr, T, H, I, E, k, 0, nullptr, false);
}

}  // namespace lg

using namespace lg;

extern "C" int lg_moe_status(const void* workspace, int T, int H, int I, int E, int k,
                             int I_shared, int* status) {
  LG_CHECK_ARG(workspace && status, "moe_status: NULL pointer");
  MoeWs w;
  carve_moe(const_cast<void*>(workspace), T, H, E > 0 ? I : 0, E, k, I_shared, &w);
  return tc_status(w.tc, T, H, E > 0 ? I : 0, I_shared, E, k, status);
}

extern "C" size_t lg_moe_workspace_bytes(int T, int H, int I, int E, int k, int I_shared) {
  if (T < 0 || H <= 0 || E < 0 || k < 0 || I < 0 || I_shared < 0) return 0;
  return carve_moe(nullptr, T, H, E > 0 ? I : 0, E, k, I_shared, nullptr);
}

extern "C" int lg_moe_experts(const void* x, int T, int H, int I, int E, int k,
                              const int32_t* inds, const void* weights,
                              float routed_scaling_factor, const uint32_t* gate_q,
                              const void* gate_s, const void* gate_b, const uint32_t* up_q,
                              const void* up_s, const void* up_b, const uint32_t* down_q,
                              const void* down_s, const void* down_b, int I_shared,
                              const uint32_t* sh_gate_q, const void* sh_gate_s,
                              const void* sh_gate_b, const uint32_t* sh_up_q,
                              const void* sh_up_s, const void* sh_up_b,
                              const uint32_t* sh_down_q, const void* sh_down_s,
                              const void* sh_down_b, int group_size, int bits, int path,
                              void* out, void* workspace, size_t workspace_bytes, void* stream) {
  const uint32_t* q[3] = {gate_q, up_q, down_q};
  const void* s[3] = {gate_s, up_s, down_s};
  const void* b[3] = {gate_b, up_b, down_b};
  const uint32_t* sq[3] = {sh_gate_q, sh_up_q, sh_down_q};
  const void* ss[3] = {sh_gate_s, sh_up_s, sh_down_s};
  const void* sb[3] = {sh_gate_b, sh_up_b, sh_down_b};
  LG_CHECK_ARG(E >= 1, "lg_moe_experts: E=%d must be >= 1 (use lg_qmlp for a dense MLP)", E);
  return moe_run(x, T, H, I, E, k, inds, weights, routed_scaling_factor, q, s, b, I_shared, sq,
                 ss, sb, group_size, bits, path, out, workspace, workspace_bytes, 0,
                 static_cast<cudaStream_t>(stream));
}

extern "C" int lg_switch_glu(const void* x, int T, int H, int I, int E, int k,
                             const int32_t* inds, const uint32_t* gate_q, const void* gate_s,
                             const void* gate_b, const uint32_t* up_q, const void* up_s,
                             const void* up_b, const uint32_t* down_q, const void* down_s,
                             const void* down_b, int group_size, int bits, int path, void* y,
                             void* workspace, size_t workspace_bytes, void* stream) {
  const uint32_t* q[3] = {gate_q, up_q, down_q};
  const void* s[3] = {gate_s, up_s, down_s};
  const void* b[3] = {gate_b, up_b, down_b};
  const uint32_t* nq[3] = {nullptr, nullptr, nullptr};
  const void* nv[3] = {nullptr, nullptr, nullptr};
  LG_CHECK_ARG(E >= 1, "lg_switch_glu: E=%d must be >= 1", E);
  return moe_run(x, T, H, I, E, k, inds, nullptr, 1.0f, q, s, b, 0, nq, nv, nv, group_size,
                 bits, path, y, workspace, workspace_bytes, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int lg_qmlp(const void* x, int T, int H, int I, const uint32_t* gate_q,
                       const void* gate_s, const void* gate_b, const uint32_t* up_q,
                       const void* up_s, const void* up_b, const uint32_t* down_q,
                       const void* down_s, const void* down_b, int group_size, int bits,
                       int path, void* out, void* workspace, size_t workspace_bytes,
                       void* stream) {
  const uint32_t* sq[3] = {gate_q, up_q, down_q};
  const void* ss[3] = {gate_s, up_s, down_s};
  const void* sb[3] = {gate_b, up_b, down_b};
  const uint32_t* nq[3] = {nullptr, nullptr, nullptr};
  const void* nv[3] = {nullptr, nullptr, nullptr};
  LG_CHECK_ARG(I > 0, "lg_qmlp: intermediate %d must be > 0", I);
  return moe_run(x, T, H, 0, 0, 0, nullptr, nullptr, 1.0f, nq, nv, nv, I, sq, ss, sb,
                 group_size, bits, path, out, workspace, workspace_bytes, 0,
                 static_cast<cudaStream_t>(stream));
}
