// Building blocks shared by the bs1 decode kernels: the RMSNorm statistics in one fixed
// order (so a norm fused into a consumer kernel gives the same bits as the standalone RMSNorm
// kernel), the warp top-k of the router, and the staging of 16-row tiles of MLX 4-bit
// matrices into shared memory with bulk copies.
#pragma once

#include <math.h>

#include "common.cuh"
#include "gemv_core.cuh"
#include "tc_ptx.cuh"

namespace lg {
using namespace tc;

// ---- RMSNorm (laguna.py:158-160; mx.fast.rms_norm) --------------------------------------

__device__ __forceinline__ float sumsq8(uint4 v) {
  const uint32_t* p = &v.x;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = __uint_as_float(p[j] << 16), b = __uint_as_float(p[j] & 0xffff0000u);
    s = __fadd_rn(s, __fmaf_rn(a, a, __fmul_rn(b, b)));
  }
  return s;
}

// 1 / sqrt(mean(h^2) + eps) of h[0, H) (bf16, H % 8 == 0), the same bits for any block size
// that is a multiple of 32: 256 virtual threads v each accumulate the 8-element chunks
// v, v + 256, ... in index order, each run of 32 virtual threads is reduced by warp_sum and
// the 8 run sums are added in order. red8: 8 floats of shared memory. Every thread calls it
// and every thread gets the result (contains __syncthreads).
__device__ __forceinline__ float block_rms_scale(const uint4* h, int H, float eps, float* red8) {
  const int nv = H / 8;
  const int nt = blockDim.x < 256 ? blockDim.x : 256;
  for (int base = 0; base < 256; base += nt) {
    if ((int)threadIdx.x < nt) {
      float ss = 0.f;
      for (int i = base + threadIdx.x; i < nv; i += 256) ss = __fadd_rn(ss, sumsq8(h[i]));
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red8[(base + threadIdx.x) >> 5] = ss;
    }
  }
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot = __fadd_rn(tot, red8[i]);
  return 1.0f / sqrtf(tot / (float)H + eps);
}

// y = bf16(bf16(h * r) * w) for 8 elements.
__device__ __forceinline__ uint4 rms_apply8(uint4 v, uint4 w, float r) {
  const uint32_t* pv = &v.x;
  const uint32_t* pw = &w.x;
  uint4 o;
  uint32_t* po = &o.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = __fmul_rn(round_bf16(__fmul_rn(__uint_as_float(pv[j] << 16), r)),
                              __uint_as_float(pw[j] << 16));
    const float b = __fmul_rn(round_bf16(__fmul_rn(__uint_as_float(pv[j] & 0xffff0000u), r)),
                              __uint_as_float(pw[j] & 0xffff0000u));
    const __nv_bfloat162 s = __floats2bfloat162_rn(a, b);
    po[j] = *reinterpret_cast<const uint32_t*>(&s);
  }
  return o;
}

// bf16(a + b) elementwise for 8 elements (the decoder's residual add).
__device__ __forceinline__ uint4 add8_bf16(uint4 a, uint4 b) {
  uint32_t* pa = &a.x;
  const uint32_t* pb = &b.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 s = __floats2bfloat162_rn(
        __fadd_rn(__uint_as_float(pa[j] << 16), __uint_as_float(pb[j] << 16)),
        __fadd_rn(__uint_as_float(pa[j] & 0xffff0000u), __uint_as_float(pb[j] & 0xffff0000u)));
    pa[j] = *reinterpret_cast<const uint32_t*>(&s);
  }
  return a;
}

// SwiGLU with the rounding points of the MLX graph (laguna.py:122): g, u -> bf16;
// silu = g * sigmoid(g) with each op rounded to bf16; h = bf16(silu * u).
__device__ __forceinline__ __nv_bfloat16 swiglu_mlx(float gv, float uv) {
  const float gr = round_bf16(gv), ur = round_bf16(uv);
  const float sig = round_bf16(1.0f / (1.0f + expf(-gr)));
  const float sl = round_bf16(gr * sig);
  return __float2bfloat16_rn(sl * ur);
}

// ---- router top-k (laguna.py:137-145) -------------------------------------------------------

__device__ __forceinline__ bool topk_better(float a, int ia, float b, int ib) {
  return (a > b) || (a == b && ia < ib);
}

constexpr int TOPK_MAXE_PER_LANE = 8;  // E <= 256

// The router's top-k in three phases, so that the middle one can run on any number of
// threads (the one-token router; the batched router uses topk_select_regs below): (1) one
// warp turns the E logits (logit(e), e < E) into scores (sigmoid, or softmax over the E
// logits) and selection keys (score + bias): keys[e], vals[e] = score;
// (2) every candidate's rank = the number of better keys under "larger first, equal keys ->
// lower index" (NaN keys are never picked); slot[rank] = e for the k best; (3) one warp reads
// the picks in rank order, adds their scores in that order and renormalises. Shared memory:
// keys [E], vals [E], slot [k] (ints).

// Phase 1 in registers: lane l holds candidates e = l + 32 j (j < NPER, 32 NPER >= E):
// sc[j] = score, key[j] = score + bias (meaningless for e >= E, which the callers skip).
template <int NPER, typename LogitFn>
__device__ __forceinline__ void topk_scores_regs(LogitFn logit, int E, const float* ebias,
                                                 int score_fn, float (&sc)[NPER],
                                                 float (&key)[NPER]) {
  const int lane = threadIdx.x & 31;
  const int nper = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    const float l = (j < nper && e < E) ? logit(e) : -INFINITY;
    sc[j] = l;
    mx = fmaxf(mx, l);
  }
  if (score_fn == LG_SCORE_SOFTMAX) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
      const int e = lane + 32 * j;
      const float v = (j < nper && e < E) ? expf(sc[j] - mx) : 0.f;
      sc[j] = v;
      sum += v;
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int j = 0; j < NPER; ++j) sc[j] = sc[j] / sum;
  } else {
#pragma unroll
    for (int j = 0; j < NPER; ++j) sc[j] = 1.0f / (1.0f + expf(-sc[j]));
  }
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    key[j] = sc[j] + ((ebias && j < nper && e < E) ? ebias[e] : 0.f);
  }
}

template <typename LogitFn>
__device__ __forceinline__ void topk_scores_warp(LogitFn logit, int E, const float* ebias,
                                                 int score_fn, float* keys, float* vals) {
  const int lane = threadIdx.x & 31;
  const int nper = (E + 31) / 32;
  float sc[TOPK_MAXE_PER_LANE], key[TOPK_MAXE_PER_LANE];
  topk_scores_regs<TOPK_MAXE_PER_LANE>(logit, E, ebias, score_fn, sc, key);
#pragma unroll
  for (int j = 0; j < TOPK_MAXE_PER_LANE; ++j) {
    const int e = lane + 32 * j;
    if (j < nper && e < E) {
      keys[e] = key[j];
      vals[e] = sc[j];
    }
  }
}

// Phases 2 and 3 for one warp in registers, after topk_scores_regs: k rounds of a warp
// arg-max over the candidates still in play, in the same total order as topk_rank (larger key
// first, equal keys -> lower index, NaN keys never picked), so the picks, their order and the
// weight sum are those of topk_rank + topk_pick_warp. A candidate is one 64-bit word: the key
// mapped to an order-preserving unsigned integer in the high half, 0xFFFF - e in the low half
// (0 = out of play). Lane j < k ends with pick j (-1 and weight 0 past the keys that are not
// NaN); its histogram count is added to hist (shared memory) when hist is not NULL.
__device__ __forceinline__ uint64_t topk_cand(float key, int e) {
  if (key != key) return 0ull;
  const uint32_t u = __float_as_uint(key == 0.f ? 0.f : key);  // -0 == +0 as in topk_better
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<uint64_t>(o) << 32) | static_cast<uint32_t>(0xFFFF - e);
}

template <int NPER>
__device__ __forceinline__ void topk_select_regs(const float (&sc)[NPER], const float (&key)[NPER],
                                                 int E, int k, int norm, int* idx, float* wt,
                                                 int* hist) {
  const int lane = threadIdx.x & 31;
  uint64_t cand[NPER];
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    cand[j] = e < E ? topk_cand(key[j], e) : 0ull;
  }
  int my_i = -1;
  float my_w = 0.f, wsum = 0.f;  // the picks' scores added in pick order
  for (int r = 0; r < k; ++r) {
    uint64_t best = 0ull;
    float bv = 0.f;
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
      if (cand[j] > best) {
        best = cand[j];
        bv = sc[j];
      }
    }
    uint64_t m = best;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const uint64_t y = __shfl_xor_sync(0xffffffffu, m, o);
      m = y > m ? y : m;
    }
    if (m == 0ull) break;  // warp-uniform: no candidate left
    const int e = 0xFFFF - static_cast<int>(m & 0xFFFFu);
    const int src = e & 31;  // candidate e lives on lane e % 32
    const float v = __shfl_sync(0xffffffffu, bv, src);
    if (lane == src) {
#pragma unroll
      for (int j = 0; j < NPER; ++j)
        if (cand[j] == m) cand[j] = 0ull;
    }
    if (lane == r) {
      my_i = e;
      my_w = v;
    }
    wsum += v;
  }
  if (lane < k) {
    if (hist && my_i >= 0) atomicAdd(&hist[my_i], 1);
    *idx = my_i;
    *wt = norm ? my_w / wsum : my_w;
  }
}

// Phase 2 for candidates e = t, t + nt, ... (t in [0, nt)); slot must hold -1 in [0, k).
__device__ __forceinline__ void topk_rank(const float* keys, int E, int k, int* slot, int t,
                                          int nt) {
  for (int e = t; e < E; e += nt) {
    const float ke = keys[e];
    if (ke != ke) continue;  // NaN keys are never picked
    int rank = 0;
#pragma unroll 8
    for (int f = 0; f < E; ++f) rank += topk_better(keys[f], f, ke, e) ? 1 : 0;
    if (rank < k) slot[rank] = e;
  }
}

// Phase 3 (one warp): lane j < k gets pick j (-1 and weight 0 if fewer keys were not NaN).
__device__ __forceinline__ void topk_pick_warp(const float* vals, const int* slot, int k,
                                               int norm, int* idx, float* wt, int* hist) {
  const int lane = threadIdx.x & 31;
  const int my_i = lane < k ? slot[lane] : -1;
  const float my_w = my_i >= 0 ? vals[my_i] : 0.f;
  if (hist && my_i >= 0) atomicAdd(&hist[my_i], 1);
  float wsum = 0.f;  // in pick order, as a sequential selection would add them
  for (int r = 0; r < k; ++r) {
    const int e = slot[r];
    wsum += e >= 0 ? vals[e] : 0.f;
  }
  if (lane < k) {
    *idx = my_i;
    *wt = norm ? my_w / wsum : my_w;
  }
}

// Router logit of one expert row for one token (a warp): dot(x, scale * code + bias) over H
// with the MLX 8-bit g64 layout, fp32, then rounded to bf16 (the quantized matmul's output).
// Lane l takes the 8-code chunks l, l + 32, ... with two accumulators (even and odd codes);
// x2: the token as bf16 pairs; w: the expert's H/4 words; s, b: its H/64 scales and biases.
// The same function serves the standalone and the fused router, so both give the same bits.
__device__ __forceinline__ float router_logit8(const __nv_bfloat162* x2, const uint32_t* w,
                                               const __nv_bfloat16* s, const __nv_bfloat16* b,
                                               int H) {
  const int lane = threadIdx.x & 31;
  float a0 = 0.f, a1 = 0.f;
  for (int c = lane; c < H / 8; c += 32) {
    const uint2 wv = *reinterpret_cast<const uint2*>(w + 2 * c);
    const uint4 xv = *reinterpret_cast<const uint4*>(x2 + 4 * c);
    const float sc = bf2f(s[c / 8]), bi = bf2f(b[c / 8]);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t word = q < 2 ? wv.x : wv.y;
      const int sh = 16 * (q & 1);
      const float w0 = fmaf(sc, code_to_f((word >> sh) & 0xffu), bi);
      const float w1 = fmaf(sc, code_to_f((word >> (sh + 8)) & 0xffu), bi);
      a0 = fmaf(__uint_as_float(xw[q] << 16), w0, a0);
      a1 = fmaf(__uint_as_float(xw[q] & 0xffff0000u), w1, a1);
    }
  }
  return round_bf16(warp_sum(a0 + a1));
}

// ---- 16-row tiles of MLX 4-bit group-64 matrices in shared memory ---------------------------
//
// Layout of one tile of a [rows, K] matrix: 16 code rows at a pitch of K/2 + 32 bytes (the
// extra 32 bytes turn the 8-row fragment reads of group_mma into conflict-free accesses),
// then scales [16][K/64] and biases [16][K/64] (bf16, unpadded). Tiles are filled with 16-byte
// asynchronous copies (cp.async) issued by every thread of the CTA.

__host__ __device__ __forceinline__ uint32_t tile_pitch(int K) { return K / 2 + 32; }
__host__ __device__ __forceinline__ uint32_t tile_sc_off(int K) { return 16 * tile_pitch(K); }
__host__ __device__ __forceinline__ uint32_t tile_bytes(int K) {
  return 16 * tile_pitch(K) + 2 * 16 * (K / 32);
}

// Check word of the staging copies (first failed check; 0 = none): [0] 1 once a copy failed,
// [1] its shared-memory offset, [2] its source address, [3] block and thread. One per
// translation unit; the one-token kernels of decode.cu use theirs, read by lg_decode_status.
static __device__ unsigned long long g_stage_check[4];

// L2 policy for data several CTAs read (keep it at normal priority).
__device__ __forceinline__ uint64_t l2_evict_normal_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Dynamic shared memory of this CTA in bytes.
__device__ __forceinline__ uint32_t dyn_smem_bytes() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}

// 16-byte asynchronous copy global -> shared (cp.async, L2 cache hint), checked: both
// addresses 16-byte aligned and the destination inside this CTA's dynamic shared memory
// [base, base + limit). A copy that fails the check is skipped and recorded.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint64_t pol,
                                           const void* base, uint32_t limit) {
  const uint32_t d = smem_u32(dst);
  const long long off = (long long)d - (long long)smem_u32(base);
  if (((reinterpret_cast<uintptr_t>(src) | d) & 15u) || off < 0 || off + 16 > (long long)limit) {
    if (atomicCAS(&g_stage_check[0], 0ull, 1ull) == 0ull) {
      g_stage_check[1] = (unsigned long long)off;
      g_stage_check[2] = (unsigned long long)reinterpret_cast<uintptr_t>(src);
      g_stage_check[3] = ((unsigned long long)blockIdx.y << 48) |
                         ((unsigned long long)blockIdx.x << 16) | threadIdx.x;
    }
    return;
  }
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most n of this thread's most recent copy groups are pending (n <= 7).
__device__ __forceinline__ void cp_async_wait(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

// This thread's share (of the whole CTA's) of the copies that fill a tile with rows
// [row0, row0 + rows) of (q, s, b), a [*, K] matrix (q rows K/8 words, s/b rows K/64 bf16).
// A partial tile (rows < 16, the last one of a matrix) stages only its codes; its readers take
// the scales and biases from global memory. sbase/slimit: this CTA's dynamic shared memory
// (the copies are checked against it). Not committed.
__device__ __forceinline__ void tile_load(uint8_t* dst, const uint32_t* q, const __nv_bfloat16* s,
                                          const __nv_bfloat16* b, int row0, int rows, int K,
                                          uint64_t pol, const void* sbase, uint32_t slimit) {
  const int cpr = K / 32;  // 16-byte chunks per code row
  const uint32_t pitch = tile_pitch(K);
  const uint8_t* qb = reinterpret_cast<const uint8_t*>(q + (size_t)row0 * (K / 8));
  for (int c = threadIdx.x; c < rows * cpr; c += blockDim.x) {
    const int rr = c / cpr, cc = c - rr * cpr;
    cp_async16(dst + rr * pitch + cc * 16, qb + (size_t)c * 16, pol, sbase, slimit);
  }
  if (rows == 16) {
    const int gpr = K / 64, sc = K / 32;  // 16-byte chunks of the tile's scales (16 * gpr * 2 B)
    const uint8_t* sb0 = reinterpret_cast<const uint8_t*>(s + (size_t)row0 * gpr);
    const uint8_t* bb0 = reinterpret_cast<const uint8_t*>(b + (size_t)row0 * gpr);
    uint8_t* d = dst + tile_sc_off(K);
    for (int c = threadIdx.x; c < 2 * sc; c += blockDim.x)
      cp_async16(d + c * 16, (c < sc ? sb0 : bb0 - sc * 16) + c * 16, pol, sbase, slimit);
  }
}

// One thread: a full tile (rows [row0, row0 + 16) of a [*, K] matrix) with bulk copies that
// complete on bar: one per code row (into the padded pitch), one for the scale block and one for
// the bias block. Not counted on bar: the caller adds tile_bulk_bytes(K) per tile to its
// expected transaction count first.
__host__ __device__ __forceinline__ uint32_t tile_bulk_bytes(int K) {
  return 16u * (K / 2) + 2u * 16u * (K / 64) * 2u;
}
__device__ __forceinline__ void tile_load_bulk(uint8_t* dst, const uint32_t* q,
                                               const __nv_bfloat16* s, const __nv_bfloat16* b,
                                               int row0, int K, uint64_t* bar) {
  const uint32_t pitch = tile_pitch(K), rb = K / 2, sbb = 16u * (K / 64) * 2u;
  const uint8_t* qb = reinterpret_cast<const uint8_t*>(q + (size_t)row0 * (K / 8));
  for (int rr = 0; rr < 16; ++rr) bulk_g2s(dst + rr * pitch, qb + (size_t)rr * rb, rb, bar);
  bulk_g2s(dst + tile_sc_off(K), s + (size_t)row0 * (K / 64), sbb, bar);
  bulk_g2s(dst + tile_sc_off(K) + sbb, b + (size_t)row0 * (K / 64), sbb, bar);
}

// One 64-group of a staged tile for a single token: the thread's A fragments (rows r, r + 8)
// from shared memory, the token's activations xa (lanes with lane/4 == 0; zero elsewhere).
__device__ __forceinline__ void tile_group(float (&d)[4], const uint8_t* tile, uint32_t pitch,
                                           int gg, int r, int c4, uint4 xa0, uint4 xa1) {
  const uint2 w0 = *reinterpret_cast<const uint2*>(tile + r * pitch + gg * 32 + c4 * 8);
  const uint2 w8 = *reinterpret_cast<const uint2*>(tile + (r + 8) * pitch + gg * 32 + c4 * 8);
  group_mma(d, w0, w8, xa0, xa1);
}

}  // namespace lg
