// Router (laguna_mlx/laguna.py:137-145) and routing plan kernels.
//
// router logits: logits[T, E] = x[T, H] . W[E, H]^T in fp32 (W fp32, or MLX 8-bit group-64
//   dequantized, whose bf16 matmul output is rounded to bf16). Three kernels: a warp per
//   (expert, token) for T <= 256 (decode, batched decode), a tensor-core kernel for fp32 W at
//   larger T (W split into three bf16 parts, so the result keeps fp32 accuracy), and a
//   CUDA-core tiled kernel otherwise.
// router_topk_kernel:   one warp per token, in registers: sigmoid (or softmax), + selection
//   bias, top-k by k rounds of a warp arg-max (larger first, equal keys -> lower index),
//   unbiased weights, renormalisation, bf16 weights; a per-CTA histogram in shared memory
//   (lane j < k adds pick j), then one global atomic per used bin and CTA.
// moe_plan_kernel:      one CTA per expert group: its exclusive offset, then an
//   order-preserving compaction of the picks of that group (warp ballot + popc prefix sums),
//   so perm is ordered by expert then pick id, independent of timing.
#include <math.h>

#include "common.cuh"
#include "decode_core.cuh"

namespace lg {

constexpr int RL_TT = 32;   // tokens per CTA
constexpr int RL_EB = 64;   // experts per CTA
constexpr int RL_KC = 32;   // H chunk

template <int GBITS>
__global__ void __launch_bounds__(256) router_logits_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, const void* __restrict__ gw,
    const __nv_bfloat16* __restrict__ gs, const __nv_bfloat16* __restrict__ gb, int E,
    float* __restrict__ logits) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
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

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}

// ---- tensor-core router logits (fp32 W, T > 256) ------------------------------------------
// x (bf16, exact) times W (fp32) with W split into three bf16 parts, hi + mid + lo = W to
// within 2^-24 relative, each product exact in the fp32 accumulator: fp32-accurate logits on
// mma.sync m16n8k16. The split is done on the B fragments in registers: each fp32 pair a
// thread loads becomes its hi, mid and lo bf16 pairs and feeds the MMAs of both of the warp's
// 16-token tiles. CTA tile 64 tokens x 64 experts, 8 warps: warp (wm, wn, kh) covers 32 tokens
// x 32 experts over k16 steps 2 kh, 2 kh + 1 of every 64-wide K chunk; the two K halves are
// added at the end. x and W chunks move by cp.async through a 4-stage ring (two CTAs fit on
// an SM); the first chunks of the static W are requested before the PDL wait.
constexpr int RX_TT = 64, RX_EB = 64, RX_KC = 64, RX_STAGES = 4;
constexpr int RX_XLD = RX_KC + 8;                  // bf16 per x row (144 B: ldmatrix rows spread)
constexpr int RX_WLD = RX_KC + 8;                  // fp32 per W row (288 B: float2 reads spread)
constexpr int RX_XB = RX_TT * RX_XLD * 2;          // 9,216 B
constexpr int RX_STAGE = RX_XB + RX_EB * RX_WLD * 4;  // 27,648 B
constexpr int RX_SMEM = RX_STAGES * RX_STAGE;      // 110,592 B

// Unchecked 16-byte copy (zero fill when !ok, reading nothing). Its callers stay in bounds by
// construction: shared offsets are stage * RX_STAGE + row * pitch + chunk * 16 with row < 64
// and chunk < 8 (x) or 16 (W), at most RX_SMEM; global rows are guarded by T and E, columns
// h0 + chunk * 8 (or 4) + 16 bytes <= H since H % 64 == 0 and h0 <= H - 64; row pitches are
// multiples of 128 bytes and the host checks 16-byte bases.
__device__ __forceinline__ void cp16_zfill(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(ok ? 16 : 0)
               : "memory");
}

// bf16x2 parts of an fp32 pair (element x in the low half): hi + mid + lo = f within 2^-24.
__device__ __forceinline__ void split3(float2 f, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
  hi = *reinterpret_cast<uint32_t*>(&h);
  const float r1x = f.x - bf_lo(hi), r1y = f.y - bf_hi(hi);
  __nv_bfloat162 m = __floats2bfloat162_rn(r1x, r1y);
  mid = *reinterpret_cast<uint32_t*>(&m);
  __nv_bfloat162 l = __floats2bfloat162_rn(r1x - bf_lo(mid), r1y - bf_hi(mid));
  lo = *reinterpret_cast<uint32_t*>(&l);
}

__global__ void __launch_bounds__(256) router_logits_rx_kernel(const __nv_bfloat16* __restrict__ x,
                                                               int T, int H,
                                                               const float* __restrict__ W, int E,
                                                               float* __restrict__ logits) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp & 1, wn = (warp >> 1) & 1, kh = warp >> 2;
  const int r = lane >> 2, c4 = lane & 3;
  const int t0 = blockIdx.y * RX_TT, e0 = blockIdx.x * RX_EB;
  const uint32_t sb = smem_u32(smem);
  const int nch = H / RX_KC;
  auto load_x = [&](int st, int h0) {  // 64 rows x 8 chunks of 16 B: 2 per thread
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + 256 * j, row = i >> 3, cc = i & 7;
      const bool ok = t0 + row < T;
      cp16_zfill(sb + st * RX_STAGE + row * (RX_XLD * 2) + cc * 16,
                 ok ? x + (size_t)(t0 + row) * H + h0 + cc * 8 : x, ok);
    }
  };
  auto load_w = [&](int st, int h0) {  // 64 rows x 16 chunks of 16 B: 4 per thread
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, row = i >> 4, cc = i & 15;
      const bool ok = e0 + row < E;
      cp16_zfill(sb + st * RX_STAGE + RX_XB + row * (RX_WLD * 4) + cc * 16,
                 ok ? W + (size_t)(e0 + row) * H + h0 + cc * 4 : W, ok);
    }
  };
  // the weight is static: its first chunks are requested while the previous kernel finishes
  for (int s = 0; s < RX_STAGES - 1; ++s)
    if (s < nch) load_w(s, s * RX_KC);
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  for (int s = 0; s < RX_STAGES - 1; ++s) {
    if (s < nch) load_x(s, s * RX_KC);
    cp_async_commit();
  }
  float acc[2][4][4];
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = acc[mi][ni][2] = acc[mi][ni][3] = 0.f;
  for (int c = 0; c < nch; ++c) {
    cp_async_wait(RX_STAGES - 2);  // chunk c has landed (this thread's copies) ...
    __syncthreads();               // ... everyone's; and the stage refilled below is free
    const int nx = c + RX_STAGES - 1;
    if (nx < nch) {
      load_w(nx % RX_STAGES, nx * RX_KC);
      load_x(nx % RX_STAGES, nx * RX_KC);
    }
    cp_async_commit();
    const uint8_t* st = smem + (c % RX_STAGES) * RX_STAGE;
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(st);
    const float* ws = reinterpret_cast<const float*>(st + RX_XB);
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int k16 = (kh * 2 + kk) * 16;
      uint32_t a[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
        ldsm_x4(&xs[(wm * 32 + mi * 16 + (lane & 15)) * RX_XLD + k16 + ((lane >> 4) << 3)],
                a[mi][0], a[mi][1], a[mi][2], a[mi][3]);
      __syncwarp();  // mma.sync.aligned: the whole warp converged
      uint32_t b[3][4][2];  // [part][n tile][k half]
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const float* wr = ws + (wn * 32 + ni * 8 + r) * RX_WLD + k16 + 2 * c4;
        split3(*reinterpret_cast<const float2*>(wr), b[0][ni][0], b[1][ni][0], b[2][ni][0]);
        split3(*reinterpret_cast<const float2*>(wr + 8), b[0][ni][1], b[1][ni][1], b[2][ni][1]);
      }
      // part-major: the 8 accumulators take turns, so an MMA never waits for the one just
      // issued (the asm statements keep their order)
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
          for (int mi = 0; mi < 2; ++mi)
            mma_bf16(acc[mi][ni], a[mi][0], a[mi][1], a[mi][2], a[mi][3], b[p][ni][0],
                     b[p][ni][1]);
    }
  }
  cp_async_wait(0);
  __syncthreads();  // the ring is free: the upper K half's sums go through it
  float* red = reinterpret_cast<float*>(smem) + (warp & 3) * 32 * 32;
  if (kh == 1) {
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni)
#pragma unroll
        for (int q = 0; q < 4; ++q) red[((mi * 4 + ni) * 4 + q) * 32 + lane] = acc[mi][ni][q];
  }
  __syncthreads();
  if (kh == 1) return;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = t0 + wm * 32 + mi * 16 + r + 8 * (q >> 1);
        const int e = e0 + wn * 32 + ni * 8 + 2 * c4 + (q & 1);
        const float v = acc[mi][ni][q] + red[((mi * 4 + ni) * 4 + q) * 32 + lane];
        if (t < T && e < E) logits[(size_t)t * E + e] = v;
      }
    }
  }
}

// ---- small-T router logits (decode): one warp per (expert, token) --------------------------
// Lanes stride over the hidden dimension two elements at a time (coalesced bf16x2 / float2
// loads) and reduce across the warp; the tokens are spread over blockIdx.y, so the T <= 256
// tokens' dot products run in parallel and each weight row is re-read from L2.
template <int GBITS>
__global__ void __launch_bounds__(256) router_logits_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, const void* __restrict__ gw,
    const __nv_bfloat16* __restrict__ gs, const __nv_bfloat16* __restrict__ gb, int E,
    float* __restrict__ logits) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (e >= E) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {  // tokens spread over blockIdx.y
    const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + (size_t)t * H);
    if (GBITS == 8) {  // the fused one-token router computes the same function
      const float v = router_logit8(xr, static_cast<const uint32_t*>(gw) + (size_t)e * (H / 4),
                                    gs + (size_t)e * (H / 64), gb + (size_t)e * (H / 64), H);
      if (lane == 0) logits[(size_t)t * E + e] = v;
      continue;
    }
    float acc = 0.f;
    for (int k2 = lane; k2 < H / 2; k2 += 32) {
      const float2 xv = __bfloat1622float2(xr[k2]);
      const float2 wv = reinterpret_cast<const float2*>(static_cast<const float*>(gw) +
                                                        (size_t)e * H)[k2];
      acc = fmaf(xv.x, wv.x, acc);
      acc = fmaf(xv.y, wv.y, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[(size_t)t * E + e] = acc;
  }
}

constexpr int TK_WARPS = 8;

// One warp per token, all in registers (NPER = candidates per lane, 32 NPER >= E).
template <int NPER>
__global__ void __launch_bounds__(TK_WARPS * 32) router_topk_kernel(
    const float* __restrict__ logits, int T, int E, const float* __restrict__ ebias, int k,
    int norm, int score_fn, int32_t* __restrict__ inds, __nv_bfloat16* __restrict__ wout,
    int32_t* __restrict__ counts) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  __shared__ int hist[256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int t = blockIdx.x * TK_WARPS + warp; t < T; t += gridDim.x * TK_WARPS) {
    const float* row = logits + (size_t)t * E;
    float sc[NPER], key[NPER];
    topk_scores_regs<NPER>([&](int e) { return row[e]; }, E, ebias, score_fn, sc, key);
    int idx = -1;
    float wt = 0.f;
    topk_select_regs<NPER>(sc, key, E, k, norm, &idx, &wt, counts ? hist : nullptr);
    if (lane < k) {
      inds[(size_t)t * k + lane] = idx;
      wout[(size_t)t * k + lane] = __float2bfloat16_rn(wt);
    }
  }
  __syncthreads();
  if (counts) {
    for (int i = threadIdx.x; i < E; i += blockDim.x)
      if (hist[i]) atomicAdd(&counts[i], hist[i]);
  }
}

// One CTA per group g in [0, G); G = E (+1 with the shared group). Expert ids outside
// [0, E) belong to no group: such picks produce no output. Each thread owns a contiguous run
// of picks, so one counting pass, one block scan and one writing pass give the group's picks
// in pick order. Every CTA writes its own offset (= valid picks of lower experts); groups with
// rows append themselves to the active list (order irrelevant; active[0] must start at 0).
__global__ void __launch_bounds__(512) moe_plan_kernel(const int32_t* __restrict__ inds, int T,
                                                       int k, int E, int with_shared,
                                                       int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ offsets,
                                                       int32_t* __restrict__ perm,
                                                       int32_t* __restrict__ active) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_total, s_before;
  const int g = blockIdx.x;
  const int P = T * k;
  const int nth = blockDim.x;
  const int per = (P + nth - 1) / nth;
  const int p0 = min(P, threadIdx.x * per), p1 = min(P, p0 + per);
  if (threadIdx.x == 0) s_before = 0;
  __syncthreads();
  int eq = 0, lt = 0;
  if ((per & 3) == 0 && (reinterpret_cast<uintptr_t>(inds) & 15) == 0) {
    for (int p = p0; p < p1; p += 4) {
      const int4 v = *reinterpret_cast<const int4*>(inds + p);
      const int e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        eq += (e[j] == g);
        lt += (e[j] >= 0 && e[j] < g);
      }
    }
  } else {
    for (int p = p0; p < p1; ++p) {
      const int e = inds[p];
      eq += (e == g);
      lt += (e >= 0 && e < g);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o);
  if ((threadIdx.x & 31) == 0 && lt) atomicAdd(&s_before, lt);
  const int off = block_excl_scan(eq, warp_tot, &s_total);  // its barriers also publish s_before
  const int before = s_before;
  if (g == E) {  // shared expert: identity rows after all valid routed picks
    for (int t = threadIdx.x; t < T; t += nth) perm[before + t] = P + t;
    if (threadIdx.x == 0) {
      counts[E] = T;
      offsets[E] = before;
      offsets[E + 1] = before + T;
      if (active && T > 0) active[1 + atomicAdd(active, 1)] = E;
    }
    return;
  }
  int j = 0;
  for (int p = p0; p < p1 && j < eq; ++p)
    if (inds[p] == g) perm[before + off + j++] = p;
  if (threadIdx.x == 0) {
    counts[g] = s_total;
    offsets[g] = before;
    if (g == E - 1 && !with_shared) offsets[E] = offsets[E + 1] = before + s_total;
    if (active && s_total > 0) active[1 + atomicAdd(active, 1)] = g;
  }
}

// ---- segmented plan for many picks (P >= PL_MIN_PICKS) ---------------------------------------
// The kernel above gives every group one CTA that scans all P picks, so its time does not
// fall with the group count (an expert-parallel owner with 16 local experts scans as many picks
// as the one-GPU block). The segmented form gives the same outputs with the scan split over
// warps: (1) every warp histograms its PL_SEG consecutive picks; (2) one CTA scans the
// (group, segment) counts in group-major order into each segment's first row per group, and
// writes counts, offsets and the active list; (3) every warp walks its segment in order and
// places each pick at its segment's running row for its group (lanes with the same group ranked
// by __match_any_sync), so perm is ordered by group, then pick id, as before.
constexpr int PL_SEG = 1024;         // picks per warp segment
constexpr int PL_WARPS = 8;          // warps per CTA in the histogram and placement kernels
constexpr int PL_MIN_PICKS = 65536;  // below this the one-CTA-per-group kernel is as fast

__host__ __device__ constexpr int pl_nseg(int P) { return (P + PL_SEG - 1) / PL_SEG; }

// cnt [nseg][E]: picks of group e in segment seg (valid routed picks only)
__global__ void __launch_bounds__(PL_WARPS * 32) plan_count_kernel(const int32_t* __restrict__ inds,
                                                                   int P, int E,
                                                                   int32_t* __restrict__ cnt) {
  pdl_wait();  // inds come from the previous kernel
  pdl_trigger();
  __shared__ int hist[PL_WARPS][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = blockIdx.x * PL_WARPS + warp;
  for (int e = lane; e < E; e += 32) hist[warp][e] = 0;
  __syncwarp();
  const int p0 = seg * PL_SEG, p1 = min(P, p0 + PL_SEG);
  for (int p = p0 + lane; p < p1; p += 32) {
    const int e = inds[p];
    if (e >= 0 && e < E) atomicAdd(&hist[warp][e], 1);
  }
  __syncwarp();
  if (p0 < P)
    for (int e = lane; e < E; e += 32) cnt[(size_t)seg * E + e] = hist[warp][e];
}

// One CTA: base[seg][e] = rows of groups < e (all segments) + rows of group e in segments
// < seg; counts, offsets (the shared group after every valid routed pick) and the active list.
__global__ void __launch_bounds__(1024) plan_scan_kernel(const int32_t* __restrict__ cnt, int nseg,
                                                         int E, int T, int with_shared,
                                                         int32_t* __restrict__ base,
                                                         int32_t* __restrict__ counts,
                                                         int32_t* __restrict__ offsets,
                                                         int32_t* __restrict__ active) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_total;
  const int N = nseg * E;  // entries in group-major order: i = e * nseg + seg
  const int per = (N + blockDim.x - 1) / blockDim.x;
  const int i0 = min(N, (int)threadIdx.x * per), i1 = min(N, i0 + per);
  int sum = 0;
  for (int i = i0; i < i1; ++i) sum += cnt[(size_t)(i % nseg) * E + i / nseg];
  int run = block_excl_scan(sum, warp_tot, &s_total);
  for (int i = i0; i < i1; ++i) {
    const int seg = i % nseg, e = i / nseg;
    base[(size_t)seg * E + e] = run;
    if (seg == 0) offsets[e] = run;
    run += cnt[(size_t)seg * E + e];
  }
  __syncthreads();  // every group's offset is written
  const int total = s_total;
  if (threadIdx.x == 0) {
    int na = 0;
    for (int e = 0; e < E; ++e) {
      const int c = (e + 1 < E ? offsets[e + 1] : total) - offsets[e];
      counts[e] = c;
      if (active && c > 0) active[1 + na++] = e;
    }
    if (with_shared) {
      counts[E] = T;
      offsets[E] = total;
      offsets[E + 1] = total + T;
      if (active && T > 0) active[1 + na++] = E;
    } else {
      offsets[E] = offsets[E + 1] = total;
    }
    if (active) active[0] = na;
  }
}

// Every warp places its segment's picks in order; the shared group's identity rows follow the
// routed picks (rows offsets[E] + t = pick P + t).
__global__ void __launch_bounds__(PL_WARPS * 32) plan_place_kernel(const int32_t* __restrict__ inds,
                                                                   int P, int E, int T,
                                                                   int with_shared,
                                                                   const int32_t* __restrict__ base,
                                                                   const int32_t* __restrict__ offsets,
                                                                   int32_t* __restrict__ perm) {
  pdl_wait();
  pdl_trigger();
  __shared__ int next[PL_WARPS][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = blockIdx.x * PL_WARPS + warp;
  const int p0 = seg * PL_SEG, p1 = min(P, p0 + PL_SEG);
  if (p0 < P) {
    for (int e = lane; e < E; e += 32) next[warp][e] = base[(size_t)seg * E + e];
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    for (int q = p0; q < p1; q += 32) {  // warp-uniform trip count
      const int p = q + lane;
      const int e = p < p1 ? inds[p] : -1;
      const bool valid = e >= 0 && e < E;
      const unsigned same = __match_any_sync(0xffffffffu, valid ? e : E + lane);
      if (valid) perm[next[warp][e] + __popc(same & lt)] = p;
      __syncwarp();  // every lane has read its group's row before the leader moves it on
      if (valid && (same & lt) == 0) next[warp][e] += __popc(same);
      __syncwarp();
    }
  }
  if (with_shared && blockIdx.x == 0) {
    const int sb = offsets[E];
    for (int t = threadIdx.x; t < T; t += blockDim.x) perm[sb + t] = P + t;
  }
}

size_t plan_scratch_bytes(int T, int k, int E) {
  const int P = T * k;
  return P >= PL_MIN_PICKS ? 2 * sizeof(int32_t) * (size_t)pl_nseg(P) * E : 0;
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
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const __nv_bfloat16* gsb = static_cast<const __nv_bfloat16*>(gate_scales);
  const __nv_bfloat16* gbb = static_cast<const __nv_bfloat16*>(gate_biases);
  const bool xa = aligned(x, 16) && aligned(gate_w, 16);
  prof_begin("router_logits", s);
  if (T <= 256) {
    // decode sizes and batched decode steps: one warp per (expert, token); the tiled kernels
    // below run one CTA per 32 tokens x 64 experts, a handful of CTAs at these sizes
    const __nv_bfloat16* nb = nullptr;
    const dim3 grid((E + 7) / 8, T);  // one (8 experts, token) per CTA: the rows come from L2
    if (gate_bits == 0)
      LG_CUDA_TRY(launch_k(router_logits_gemv_kernel<0>, grid, dim3(256), 0, s, xb, T, H, gate_w,
                           nb, nb, E, logits));
    else
      LG_CUDA_TRY(launch_k(router_logits_gemv_kernel<8>, grid, dim3(256), 0, s, xb, T, H, gate_w,
                           gsb, gbb, E, logits));
  } else if (gate_bits == 0 && xa) {
    dim3 g((E + RX_EB - 1) / RX_EB, (T + RX_TT - 1) / RX_TT);
    LG_CUDA_TRY(cudaFuncSetAttribute(router_logits_rx_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, RX_SMEM));
    LG_CUDA_TRY(launch_k(router_logits_rx_kernel, g, dim3(256), (size_t)RX_SMEM, s, xb, T, H,
                         static_cast<const float*>(gate_w), E, logits));
  } else {
    dim3 g1((E + RL_EB - 1) / RL_EB, (T + RL_TT - 1) / RL_TT);
    const __nv_bfloat16* nb = nullptr;
    if (gate_bits == 0)
      LG_CUDA_TRY(launch_k(router_logits_kernel<0>, g1, dim3(256), 0, s, xb, T, H, gate_w, nb, nb,
                           E, logits));
    else
      LG_CUDA_TRY(launch_k(router_logits_kernel<8>, g1, dim3(256), 0, s, xb, T, H, gate_w, gsb,
                           gbb, E, logits));
  }
  prof_end("router_logits", s);
  LG_LAUNCH_CHECK("router_logits");
  int blocks = (T + TK_WARPS - 1) / TK_WARPS;
  if (blocks > 1184) blocks = 1184;
  prof_begin("router_topk", s);
  {
    auto kern = E <= 32 ? router_topk_kernel<1> : E <= 64 ? router_topk_kernel<2>
              : E <= 128 ? router_topk_kernel<4> : router_topk_kernel<8>;
    LG_CUDA_TRY(launch_k(kern, dim3(blocks), dim3(TK_WARPS * 32), 0, s,
                         static_cast<const float*>(logits), T, E, e_bias, k, norm_topk_prob,
                         score_fn, inds, static_cast<__nv_bfloat16*>(weights), counts));
  }
  prof_end("router_topk", s);
  LG_LAUNCH_CHECK("router_topk");
  return LG_OK;
}

namespace lg {
// Host-side plan launch shared with the MoE orchestration. active: int32 [1 + E + 1].
int launch_plan(const int32_t* inds, int T, int k, int E, int with_shared, int32_t* counts,
                int32_t* offsets, int32_t* perm, int32_t* active, cudaStream_t s,
                int32_t* scratch) {
  int G = E + (with_shared ? 1 : 0);
  if (G == 0) return LG_OK;
  const int P = T * k;
  if (scratch && P >= PL_MIN_PICKS && E > 0 && E <= 256) {  // segmented form
    const int nseg = pl_nseg(P);
    int32_t* cnt = scratch;
    int32_t* base = scratch + (size_t)nseg * E;
    const int blocks = (nseg + PL_WARPS - 1) / PL_WARPS;
    prof_begin("plan", s);
    LG_CUDA_TRY(launch_k(plan_count_kernel, dim3(blocks), dim3(PL_WARPS * 32), 0, s, inds, P, E,
                         cnt));
    LG_CUDA_TRY(launch_k(plan_scan_kernel, dim3(1), dim3(1024), 0, s,
                         static_cast<const int32_t*>(cnt), nseg, E, T, with_shared, base, counts,
                         offsets, active));
    LG_CUDA_TRY(launch_k(plan_place_kernel, dim3(blocks), dim3(PL_WARPS * 32), 0, s, inds, P, E,
                         T, with_shared, static_cast<const int32_t*>(base),
                         static_cast<const int32_t*>(offsets), perm));
    prof_end("plan", s);
    LG_LAUNCH_CHECK("moe_plan_segmented");
    return LG_OK;
  }
  if (active) LG_CUDA_TRY(cudaMemsetAsync(active, 0, sizeof(int32_t), s));
  prof_begin("plan", s);
  LG_CUDA_TRY(launch_k(moe_plan_kernel, dim3(G), dim3(512), 0, s, inds, T, k, E, with_shared,
                       counts, offsets, perm, active));
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
                     static_cast<cudaStream_t>(stream), nullptr);
}
