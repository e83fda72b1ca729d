// Router (laguna_mlx/laguna.py:137-145) and routing plan kernels.
//
// router_logits_kernel: logits[T, E] = x[T, H] . W[E, H]^T in fp32 (W fp32, or MLX 8-bit
//   group-64 dequantized while staging, whose bf16 matmul output is rounded to bf16).
// router_topk_kernel:   one warp per token: sigmoid (or softmax), + selection bias, top-k by
//   repeated warp arg-max (larger first, equal keys -> lower index), unbiased weights,
//   renormalisation, bf16 weights; a per-CTA histogram in shared memory (the warp's winning
//   lane-0 adds one count per pick), then one global atomic per used bin and CTA.
// moe_plan_kernel:      one CTA per expert group: its exclusive offset, then an
//   order-preserving compaction of the picks of that group (warp ballot + popc prefix sums),
//   so perm is ordered by expert then pick id, independent of timing.
#include <math.h>

#include "common.cuh"

namespace lg {

constexpr int RL_TT = 32;   // tokens per CTA
constexpr int RL_EB = 64;   // experts per CTA
constexpr int RL_KC = 32;   // H chunk

template <int GBITS>
__global__ void __launch_bounds__(256) router_logits_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, const void* __restrict__ gw,
    const __nv_bfloat16* __restrict__ gs, const __nv_bfloat16* __restrict__ gb, int E,
    float* __restrict__ logits) {
  __shared__ float xs[RL_KC][RL_TT + 1];
  __shared__ float ws[RL_KC][RL_EB + 1];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.y * RL_TT;
  const int e0 = blockIdx.x * RL_EB;
  const int ty = tid / 16, tx = tid % 16;  // thread owns tokens ty*2+{0,1}, experts tx*4+{0..3}
  float acc[2][4] = {};
  for (int h0 = 0; h0 < H; h0 += RL_KC) {
    // stage x chunk: RL_TT x RL_KC
    for (int i = tid; i < RL_TT * RL_KC; i += 256) {
      int tt = i / RL_KC, kk = i % RL_KC;
      int t = t0 + tt;
      xs[kk][tt] = (t < T) ? bf2f(x[(size_t)t * H + h0 + kk]) : 0.f;
    }
    // stage W chunk: RL_EB x RL_KC
    for (int i = tid; i < RL_EB * RL_KC; i += 256) {
      int ee = i / RL_KC, kk = i % RL_KC;
      int e = e0 + ee;
      float v = 0.f;
      if (e < E) {
        int h = h0 + kk;
        if (GBITS == 0) {
          v = static_cast<const float*>(gw)[(size_t)e * H + h];
        } else {
          uint32_t w = static_cast<const uint32_t*>(gw)[(size_t)e * (H / 4) + h / 4];
          uint32_t c = (w >> (8 * (h & 3))) & 0xffu;
          float s = bf2f(gs[(size_t)e * (H / 64) + h / 64]);
          float b = bf2f(gb[(size_t)e * (H / 64) + h / 64]);
          v = fmaf(s, code_to_f(c), b);
        }
      }
      ws[kk][ee] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < RL_KC; ++kk) {
      float xv0 = xs[kk][ty * 2], xv1 = xs[kk][ty * 2 + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float wv = ws[kk][tx * 4 + j];
        acc[0][j] = fmaf(xv0, wv, acc[0][j]);
        acc[1][j] = fmaf(xv1, wv, acc[1][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    int t = t0 + ty * 2 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int e = e0 + tx * 4 + j;
      if (e < E) {
        float v = acc[i][j];
        if (GBITS == 8) v = round_bf16(v);  // quantized matmul output is bf16 (laguna.py:138)
        logits[(size_t)t * E + e] = v;
      }
    }
  }
}

__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  return (a > b) || (a == b && ia < ib);
}

constexpr int TK_WARPS = 8;
constexpr int MAXE_PER_LANE = 8;  // E <= 256

__global__ void __launch_bounds__(TK_WARPS * 32) router_topk_kernel(
    const float* __restrict__ logits, int T, int E, const float* __restrict__ ebias, int k,
    int norm, int score_fn, int32_t* __restrict__ inds, __nv_bfloat16* __restrict__ wout,
    int32_t* __restrict__ counts) {
  __shared__ int hist[256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int nper = (E + 31) / 32;
  for (int t = blockIdx.x * TK_WARPS + warp; t < T; t += gridDim.x * TK_WARPS) {
    float sc[MAXE_PER_LANE], sl[MAXE_PER_LANE];
    const float* row = logits + (size_t)t * E;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < MAXE_PER_LANE; ++j) {
      int e = lane + 32 * j;
      float l = (j < nper && e < E) ? row[e] : -INFINITY;
      sc[j] = l;
      mx = fmaxf(mx, l);
    }
    if (score_fn == LG_SCORE_SOFTMAX) {
      mx = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < MAXE_PER_LANE; ++j) {
        int e = lane + 32 * j;
        float v = (j < nper && e < E) ? expf(sc[j] - mx) : 0.f;
        sc[j] = v;
        sum += v;
      }
      sum = warp_sum(sum);
#pragma unroll
      for (int j = 0; j < MAXE_PER_LANE; ++j) sc[j] = sc[j] / sum;
    } else {
#pragma unroll
      for (int j = 0; j < MAXE_PER_LANE; ++j) sc[j] = 1.0f / (1.0f + expf(-sc[j]));
    }
#pragma unroll
    for (int j = 0; j < MAXE_PER_LANE; ++j) {
      int e = lane + 32 * j;
      bool ok = (j < nper && e < E);
      sl[j] = ok ? sc[j] + (ebias ? ebias[e] : 0.f) : -INFINITY;
      if (!ok) sc[j] = 0.f;
    }
    unsigned taken = 0;  // bit j: expert lane + 32 j already selected
    float my_w = 0.f, wsum = 0.f;
    int my_i = -1;
    for (int r = 0; r < k; ++r) {
      // local best among untaken
      float bv = -INFINITY, bs = 0.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < MAXE_PER_LANE; ++j) {
        int e = lane + 32 * j;
        if (j < nper && e < E && !((taken >> j) & 1u) && better(sl[j], e, bv, bi)) {
          bv = sl[j];
          bs = sc[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        float os = __shfl_xor_sync(0xffffffffu, bs, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bs = os;
          bi = oi;
        }
      }
      const bool valid = bi >= 0 && bi < E;  // false only if every candidate is NaN
      if (valid && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (lane == r) {
        my_i = valid ? bi : -1;
        my_w = valid ? bs : 0.f;
      }
      wsum += valid ? bs : 0.f;
      if (lane == 0 && valid) atomicAdd(&hist[bi], 1);  // one shared atomic per pick
    }
    if (lane < k) {
      float w = my_w;
      if (norm) w = w / wsum;
      inds[(size_t)t * k + lane] = my_i;
      wout[(size_t)t * k + lane] = __float2bfloat16_rn(w);
    }
  }
  __syncthreads();
  if (counts) {
    for (int i = threadIdx.x; i < E; i += blockDim.x)
      if (hist[i]) atomicAdd(&counts[i], hist[i]);
  }
}

// One CTA per group g in [0, G); G = E (+1 with the shared group). Expert ids outside
// [0, E) belong to no group: such picks produce no output.
__global__ void __launch_bounds__(512) moe_plan_kernel(const int32_t* __restrict__ inds, int T,
                                                       int k, int E, int with_shared,
                                                       int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ offsets,
                                                       int32_t* __restrict__ perm,
                                                       int32_t* __restrict__ active) {
  __shared__ int warp_tot[16];
  __shared__ int s_base;
  __shared__ int cnt[257];
  const int g = blockIdx.x;
  const int G = E + (with_shared ? 1 : 0);
  const int P = T * k;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  if (g == E) {
    // shared expert: identity rows T*k + t, after every routed group
    for (int t = threadIdx.x; t < T; t += blockDim.x) perm[P + t] = P + t;
    if (threadIdx.x == 0) counts[E] = T;
  } else {
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    // offset of group g = number of valid picks with expert < g
    int before = 0;
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
      int e = inds[p];
      before += (e >= 0 && e < g) ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
    if (lane == 0) atomicAdd(&s_base, before);
    __syncthreads();
    const int base = s_base;
    int running = 0;
    for (int p0 = 0; p0 < P; p0 += blockDim.x) {
      int p = p0 + threadIdx.x;
      bool f = (p < P) && (inds[p] == g);
      unsigned m = __ballot_sync(0xffffffffu, f);
      if (lane == 0) warp_tot[warp] = __popc(m);
      __syncthreads();
      int wpre = 0, tot = 0;
      for (int w = 0; w < nwarps; ++w) {
        int c = warp_tot[w];
        if (w < warp) wpre += c;
        tot += c;
      }
      if (f) perm[base + running + wpre + __popc(m & ((1u << lane) - 1u))] = p;
      running += tot;
      __syncthreads();
    }
    if (threadIdx.x == 0) counts[g] = running;
  }
  if (g == 0) {
    // CTA 0 also writes the offsets (and the active-group list); it recounts every group
    // itself so that it does not depend on the other CTAs.
    for (int i = threadIdx.x; i < 257; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
      int e = inds[p];
      if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      if (with_shared) cnt[E] = T;
      int acc = 0, na = 0;
      for (int i = 0; i < G; ++i) {
        offsets[i] = acc;
        acc += cnt[i];
        if (active && cnt[i] > 0) active[1 + na++] = i;
      }
      offsets[G] = acc;
      if (!with_shared) offsets[E + 1] = acc;
      if (active) active[0] = na;
    }
  }
}

}  // namespace lg

using namespace lg;

extern "C" int lg_router_topk(const void* x, int T, int H, const void* gate_w,
                              const void* gate_scales, const void* gate_biases, int gate_bits,
                              const float* e_bias, int E, int k, int norm_topk_prob,
                              int score_fn, int32_t* inds, void* weights, float* logits,
                              int32_t* counts, void* stream) {
  LG_CHECK_ARG(T >= 0 && H > 0 && E > 0, "router: bad sizes T=%d H=%d E=%d", T, H, E);
  LG_CHECK_ARG(E <= 256, "router: E=%d > 256 is not supported", E);
  LG_CHECK_ARG(k >= 1 && k <= E && k <= 32, "router: k=%d must be in [1, min(E, 32)]", k);
  LG_CHECK_ARG(H % 64 == 0, "router: hidden %d must be a multiple of 64", H);
  LG_CHECK_ARG(gate_bits == 0 || gate_bits == 8, "router: gate_bits %d not in {0, 8}",
               gate_bits);
  LG_CHECK_ARG(score_fn == LG_SCORE_SIGMOID || score_fn == LG_SCORE_SOFTMAX,
               "router: score_fn %d", score_fn);
  LG_CHECK_ARG(x && gate_w && inds && weights, "router: NULL pointer");
  LG_CHECK_ARG(gate_bits == 0 || (gate_scales && gate_biases), "router: 8-bit gate needs scales/biases");
  LG_CHECK_ARG(logits != nullptr, "router: logits buffer [T, E] fp32 is required (scratch)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (counts) LG_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, s));
  if (T == 0) return LG_OK;
  dim3 g1((E + RL_EB - 1) / RL_EB, (T + RL_TT - 1) / RL_TT);
  prof_begin("router_logits", s);
  if (gate_bits == 0)
    router_logits_kernel<0><<<g1, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), T, H,
                                               gate_w, nullptr, nullptr, E, logits);
  else
    router_logits_kernel<8><<<g1, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), T, H, gate_w,
        static_cast<const __nv_bfloat16*>(gate_scales),
        static_cast<const __nv_bfloat16*>(gate_biases), E, logits);
  prof_end("router_logits", s);
  LG_LAUNCH_CHECK("router_logits");
  int blocks = (T + TK_WARPS - 1) / TK_WARPS;
  if (blocks > 1184) blocks = 1184;
  prof_begin("router_topk", s);
  router_topk_kernel<<<blocks, TK_WARPS * 32, 0, s>>>(logits, T, E, e_bias, k, norm_topk_prob,
                                                      score_fn, inds,
                                                      static_cast<__nv_bfloat16*>(weights), counts);
  prof_end("router_topk", s);
  LG_LAUNCH_CHECK("router_topk");
  return LG_OK;
}

namespace lg {
// Host-side plan launch shared with the MoE orchestration. active: int32 [1 + E + 1].
int launch_plan(const int32_t* inds, int T, int k, int E, int with_shared, int32_t* counts,
                int32_t* offsets, int32_t* perm, int32_t* active, cudaStream_t s) {
  int G = E + (with_shared ? 1 : 0);
  if (G == 0) return LG_OK;
  prof_begin("plan", s);
  moe_plan_kernel<<<G, 512, 0, s>>>(inds, T, k, E, with_shared, counts, offsets, perm, active);
  prof_end("plan", s);
  LG_LAUNCH_CHECK("moe_plan");
  return LG_OK;
}
}  // namespace lg

extern "C" int lg_moe_plan(const int32_t* inds, int T, int k, int E, int with_shared,
                           int32_t* counts, int32_t* offsets, int32_t* perm, void* stream) {
  LG_CHECK_ARG(T >= 0 && k >= 0 && E >= 0 && E <= 256, "plan: bad sizes");
  LG_CHECK_ARG(counts && offsets && perm, "plan: NULL pointer");
  LG_CHECK_ARG(T * k == 0 || inds, "plan: NULL inds");
  return launch_plan(inds, T, k, E, with_shared, counts, offsets, perm, nullptr,
                     static_cast<cudaStream_t>(stream));
}
