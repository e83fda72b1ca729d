// The attention prologue of one (token, head slot), shared by the standalone prologue kernel
// (decoder.cu) and the q/k/v/g projection GEMV that finishes each head itself (decode.cu), so
// both give the same bits.
#pragma once

#include <math.h>

#include "common.cuh"

namespace lg {

// ---------------------------------------------------------------------------------------
// Attention prologue (laguna.py:94-104): from the fused projection row
// [q (Hq*D) | k (Hkv*D) | v (Hkv*D) | g (Hq or Hq*D)] of token t at position p = pos + t:
//   q = rope(bf16(rmsnorm(q_h, qn_w)), p)  -> q_out [Hq, T, D]
//   k = rope(bf16(rmsnorm(k_h, kn_w)), p)  -> k_cache [Hkv, cap, D] row p
//   v                                       -> v_cache row p
//   gate = bf16(softplus(float(g)))         -> gate_out [T, Hq or Hq*D]
// RoPE is the non-interleaved form (mx.fast.rope traditional=False) on the first R dims: pairs
// (i, i + R/2), fp32 angles, one bf16 rounding, dims past R unchanged. Default: R = D and
// inv_freq_i = theta^(-2i/D) computed in the kernel; otherwise (partial rotary, YaRN,
// laguna.py:62-72) the caller's inv_freq table [R/2] and, when mscale != 1, the rotated dims
// scaled by mscale and rounded to bf16 first (mlx-lm's YaRN layer).
// Cache row of position p: p - row0, or p mod ring for a sliding-window ring buffer.
// ---------------------------------------------------------------------------------------
struct PrepArgs {
  const __nv_bfloat16* qkvg;
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const int* pos_dev;
  int pos_host, T, Hq, Hkv, D, cap, gate_per_head;
  float eps, log2_theta;
  const float* inv_freq;  // [rot_half] (null: the default theta^(-2i/D), all D dims rotated)
  int rot_half;           // R / 2: a multiple of 32 (0: D / 2)
  float mscale;           // YaRN attention factor on the rotated dims (1: none)
  int ring;               // > 0: cache row = position mod ring (sliding window)
  int row0;               // linear caches: cache row = position - row0
  // 0: the T tokens are consecutive positions of one sequence (pos + t); 1: token t is the
  // newest token of stream t, at position pos_dev[t] (or pos_host), and the caches hold T
  // streams [T, Hkv, cap, D] (batched decode)
  int streams;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  __nv_bfloat16* gate_out;
  // 8-bit g64 cache destination instead of k_cache / v_cache (null: bf16 cache): words
  // [Hkv, cap, D/4], scales and biases [Hkv, cap, D/64]
  uint32_t* kq;
  __nv_bfloat16 *ks, *kb;
  uint32_t* vq;
  __nv_bfloat16 *vs, *vb;
};

// Host side: the RoPE and cache-row extension of a prologue (partial rotary / YaRN table,
// sliding-window ring). rot_dims 0 = all D dims with the default frequencies (inv_freq NULL);
// otherwise a multiple of 64 up to D with a table of rot_dims / 2 frequencies.
inline int prep_extend(PrepArgs* a, int D, const float* inv_freq, int rot_dims, float mscale,
                       int ring, int row0, const char* who) {
  if (rot_dims == 0) rot_dims = D;
  LG_CHECK_ARG(rot_dims > 0 && rot_dims <= D && rot_dims % 64 == 0,
               "%s: rotary dims %d must be a multiple of 64 up to head_dim %d", who, rot_dims, D);
  LG_CHECK_ARG(inv_freq || (rot_dims == D && mscale == 1.0f),
               "%s: partial rotary or YaRN needs a frequency table", who);
  LG_CHECK_ARG(ring >= 0 && row0 >= 0, "%s: ring %d / row0 %d", who, ring, row0);
  a->inv_freq = inv_freq;
  a->rot_half = rot_dims / 2;
  a->mscale = mscale;
  a->ring = ring;
  a->row0 = row0;
  return LG_OK;
}

// Quantize the row that one warp holds (lane l: elements l + 32 k, k < 2P, so element k's group
// of 64 is k / 2) into cache row `row` of an 8-bit g64 packed cache; the arithmetic of
// quantize_rows_kernel (quant.cu). sb: 64 P bytes of the warp's own shared memory.
template <int P>
__device__ __forceinline__ void quantize_row8_warp(const float (&v)[2 * P], size_t row,
                                                   uint32_t* q, __nv_bfloat16* sc,
                                                   __nv_bfloat16* bi, uint8_t* sb) {
  constexpr int D = 64 * P;
  const int l = threadIdx.x & 31;
  float s[P], b[P];
#pragma unroll
  for (int g = 0; g < P; ++g) {
    float lo = fminf(v[2 * g], v[2 * g + 1]), hi = fmaxf(v[2 * g], v[2 * g + 1]);
    warp_minmax(lo, hi);
    __nv_bfloat16 sbf, bbf;
    quant_group_params(lo, hi, 255.f, &sbf, &bbf);
    if (l == g) {
      sc[row * P + g] = sbf;
      bi[row * P + g] = bbf;
    }
    s[g] = bf2f(sbf);
    b[g] = bf2f(bbf);
  }
#pragma unroll
  for (int k = 0; k < 2 * P; ++k)
    sb[l + 32 * k] = (uint8_t)quant_code(v[k], s[k / 2], b[k / 2], 255.f);
  __syncwarp();
  const uint32_t* w = reinterpret_cast<const uint32_t*>(sb);  // byte j of word i: element 4i+j
#pragma unroll
  for (int i = l; i < D / 4; i += 32) q[row * (D / 4) + i] = w[i];
  __syncwarp();
}

// The output gate bf16(softplus(float(g))) (laguna.py:105-106), softplus = logaddexp(g, 0).
__device__ __forceinline__ __nv_bfloat16 prep_gate(float g) {
  return __float2bfloat16_rn(fmaxf(g, 0.f) + log1pf(expf(-fabsf(g))));
}

// RoPE on the first 64 PR dims from the caller's frequency table: lane chunks j and j + PR
// (elements l + 32 j and l + 32 (j + PR)) are the pair (i, i + 32 PR).
template <int P, int PR>
__device__ __forceinline__ void rope_table(float (&x)[2 * P], const PrepArgs& a, int pos, int l) {
#pragma unroll
  for (int j = 0; j < PR; ++j) {
    float sn, cs;
    sincosf((float)pos * a.inv_freq[l + 32 * j], &sn, &cs);
    float n0 = x[j], n1 = x[j + PR];
    if (a.mscale != 1.0f) {
      n0 = round_bf16(n0 * a.mscale);
      n1 = round_bf16(n1 * a.mscale);
    }
    x[j] = n0 * cs - n1 * sn;
    x[j + PR] = n0 * sn + n1 * cs;
  }
}

// One (token t, head slot) of the prologue, by one warp: slots [0, Hq) q heads, [Hq, Hq+Hkv)
// k heads, [Hq+Hkv, Hq+2Hkv) v heads; D = 64 P. Lane l holds elements l + 32 k (k < 2P), so the
// rotary pairs (i, i + D/2) are its own slots (k, k + P) and no barrier is needed. write_gate: a
// q head also writes its output gate(s). The projection row is read through L2 (it may come
// from other CTAs of the same launch). sb: 64 P bytes of the warp's own shared memory.
template <int P>
__device__ __forceinline__ void prep_head_warp(const PrepArgs& a, int t, int slot,
                                               bool write_gate, uint8_t* sb) {
  constexpr int D = 64 * P;
  const int l = threadIdx.x & 31;
  const int pos = a.streams ? (a.pos_dev ? a.pos_dev[t] : a.pos_host)
                            : (a.pos_dev ? a.pos_dev[0] : a.pos_host) + t;
  const int crow = a.ring > 0 ? pos % a.ring : pos - a.row0;  // the position's cache row
  const size_t srow = a.streams ? (size_t)t * a.Hkv * a.cap : 0;  // the stream's first row
  const int row_stride = (a.Hq + 2 * a.Hkv) * D + (a.gate_per_head ? a.Hq : a.Hq * D);
  const __nv_bfloat16* row = a.qkvg + (size_t)t * row_stride;
  float x[2 * P];
  if (slot >= a.Hq + a.Hkv) {  // v: into the cache as it is
    const int h = slot - a.Hq - a.Hkv;
    const __nv_bfloat16* src = row + (a.Hq + a.Hkv + h) * D;
    if (crow < 0 || crow >= a.cap) return;
    if (a.vq) {
#pragma unroll
      for (int k = 0; k < 2 * P; ++k) x[k] = bf2f(__ldcg(src + l + 32 * k));
      quantize_row8_warp<P>(x, srow + (size_t)h * a.cap + crow, a.vq, a.vs, a.vb, sb);
    } else {
      __nv_bfloat16* dst = a.v_cache + (srow + (size_t)h * a.cap + crow) * D;
#pragma unroll
      for (int k = 0; k < 2 * P; ++k) dst[l + 32 * k] = __ldcg(src + l + 32 * k);
    }
    return;
  }
  const bool is_q = slot < a.Hq;
  const int h = is_q ? slot : slot - a.Hq;
  const __nv_bfloat16* src = row + (is_q ? h : a.Hq + h) * D;
  const __nv_bfloat16* nw = is_q ? a.qn_w : a.kn_w;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 2 * P; ++k) {
    x[k] = bf2f(__ldcg(src + l + 32 * k));
    ss += x[k] * x[k];
  }
  ss = warp_sum(ss);
  const float rn = 1.0f / sqrtf(ss / (float)D + a.eps);
#pragma unroll
  for (int k = 0; k < 2 * P; ++k) x[k] = round_bf16(round_bf16(x[k] * rn) * bf2f(nw[l + 32 * k]));
  if (!a.inv_freq) {  // default RoPE over all D dims
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int i = l + 32 * j;
      const float inv_freq = exp2f(-(float)(2 * i) / (float)D * a.log2_theta);
      float sn, cs;
      sincosf((float)pos * inv_freq, &sn, &cs);
      const float n0 = x[j], n1 = x[j + P];
      x[j] = n0 * cs - n1 * sn;
      x[j + P] = n0 * sn + n1 * cs;
    }
  } else {  // the first 2 * rot_half dims with table frequencies
    const int Pr = a.rot_half / 32;
    if (Pr == 1) rope_table<P, 1>(x, a, pos, l);
    if constexpr (P >= 2) if (Pr == 2) rope_table<P, 2>(x, a, pos, l);
    if constexpr (P >= 4) if (Pr == 4) rope_table<P, 4>(x, a, pos, l);
  }
  if (is_q) {
    // q_out: [Hq, T, D], or [T, Hq, D] for streams (the batched attention's layout)
    __nv_bfloat16* dst = a.q_out + (a.streams ? (size_t)t * a.Hq + h : (size_t)h * a.T + t) * D;
#pragma unroll
    for (int k = 0; k < 2 * P; ++k) dst[l + 32 * k] = __float2bfloat16_rn(x[k]);
    if (write_gate) {
      const __nv_bfloat16* g = row + (a.Hq + 2 * a.Hkv) * D;
      if (a.gate_per_head) {
        if (l == 0) a.gate_out[(size_t)t * a.Hq + h] = prep_gate(bf2f(__ldcg(g + h)));
      } else {
        __nv_bfloat16* go = a.gate_out + (size_t)t * a.Hq * D + (size_t)h * D;
#pragma unroll
        for (int k = 0; k < 2 * P; ++k)
          go[l + 32 * k] = prep_gate(bf2f(__ldcg(g + h * D + l + 32 * k)));
      }
    }
  } else if (crow >= 0 && crow < a.cap) {
    if (a.kq) {
#pragma unroll
      for (int k = 0; k < 2 * P; ++k) x[k] = round_bf16(x[k]);
      quantize_row8_warp<P>(x, srow + (size_t)h * a.cap + crow, a.kq, a.ks, a.kb, sb);
    } else {
      __nv_bfloat16* dst = a.k_cache + (srow + (size_t)h * a.cap + crow) * D;
#pragma unroll
      for (int k = 0; k < 2 * P; ++k) dst[l + 32 * k] = __float2bfloat16_rn(x[k]);
    }
  }
}

// prep_head_warp for the head size a.D (64, 128 or 256; the hosts check it).
__device__ __forceinline__ void prep_head(const PrepArgs& a, int t, int slot, bool write_gate,
                                          uint8_t* sb) {
  if (a.D == 128)
    prep_head_warp<2>(a, t, slot, write_gate, sb);
  else if (a.D == 64)
    prep_head_warp<1>(a, t, slot, write_gate, sb);
  else
    prep_head_warp<4>(a, t, slot, write_gate, sb);
}

}  // namespace lg
