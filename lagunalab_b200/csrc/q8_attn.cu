// Fused split-KV decode attention over an MLX 8-bit group-64 KV cache
// (laguna_mlx/q8_attn.py:17-130), rebuilt for B200.
//
// Work split: grid (splits, kv heads, batch); each CTA owns a contiguous key range of one kv
// head and its whole GQA group (up to 16 query heads), 4 warps, each warp walks 16-key tiles.
// The last CTA of each (batch, kv head) to finish merges the per-CTA partials (log-sum-exp
// merge of q8_attn.py:127-130) and writes the bf16 output, so one launch does everything.
// Completion is counted with one atomic per CTA; nothing waits on another CTA.
//
// Arithmetic: both products run on the tensor cores (mma.sync m16n8k16, fp16 in, fp32 accum)
// on the raw 8-bit codes, which are exact in fp16 (0x6400 | c) - 1024. The affine
// dequantisation value = scale * code + bias (q8_attn.py:50, :55) is folded in:
//   score(h, t) = sum_g ks[t,g] * (q_h . code_k[t, g]) + kb[t,g] * sum(q_h[g])
//   out(h, d)   = sum_t (p[h,t] * vs[t,g(d)]) * code_v[t, d] + sum_t p[h,t] * vb[t,g(d)]
// so K and V are never dequantized element by element. Scores are kept in the log2 domain
// (q pre-scaled by scale * log2(e)); the softmax and the partials are fp32.
//
// Fragment mapping (S = Q K^T, M = query heads padded to 16, N = 8 keys, K = 16 dims):
// the head dimension is contracted, so it is permuted inside each 16-dim k-block: thread
// (row r = lane/4, c4 = lane%4) takes for k-block kb (group g = kb/4, word wi = kb%4) the
// code word 16g + 4c4 + wi of its key (two uint4 loads per key row per thread), and the query
// uses the same permutation. V is converted to fp16 codes in a swizzled shared-memory tile and
// read with ldmatrix.trans for the P.V product.
#include <math.h>

#include "common.cuh"

namespace lg {

constexpr int QA_WARPS = 4;
constexpr int QA_D = 128;
constexpr float QA_PSCALE = 256.0f;  // keeps p * vs in fp16's normal range

__device__ __forceinline__ uint32_t prmt32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// fp16x2 {code(byte i0), code(byte i1)} from a packed word, exact.
__device__ __forceinline__ uint32_t codes_h2(uint32_t w, uint32_t sel) {
  uint32_t v = prmt32(w, 0x64646464u, sel), r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64006400u));
  return r;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ float bfl(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bfh(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

struct Q8Args {
  const __nv_bfloat16* q;  // [B, Hq, D]
  const uint32_t* kq;      // [B, Hkv, cap, 32]
  const __nv_bfloat16* ks;  // [B, Hkv, cap, 2]
  const __nv_bfloat16* kb;
  const uint32_t* vq;
  const __nv_bfloat16* vs;
  const __nv_bfloat16* vb;
  int B, Hq, Hkv, G, cap, n, kpc, nsplit;
  float qscale;            // scale * log2(e)
  float* part;             // [B, Hkv, nsplit, G, D + 2]
  int* counters;           // [B * Hkv]
  __nv_bfloat16* out;      // [B, Hq, D]
};

__global__ void __launch_bounds__(QA_WARPS * 32) q8_decode_kernel(Q8Args a) {
  __shared__ __align__(16) uint16_t vtile[QA_WARPS][16 * QA_D];
  __shared__ float s_m[QA_WARPS][16], s_l[QA_WARPS][16];
  __shared__ float s_acc[16][QA_D + 4];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c4 = lane & 3;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G;
  const int k_begin = split * a.kpc;
  const int k_end = min(k_begin + a.kpc, a.n);
  const size_t head_row0 = ((size_t)b * a.Hkv + hk) * a.cap;

  // ---- query fragments (A of S = Q K^T), rows r and r + 8 of the padded group ----
  uint32_t qa[8][4];
  float qsum[2][2];  // [group][row r / r+8]
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int h = r + 8 * rr;
    const bool hv = h < G;
    const __nv_bfloat16* qrow = a.q + ((size_t)b * a.Hq + hk * G + (hv ? h : 0)) * QA_D;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      float s = 0.f;
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        const int d0 = 64 * g + 16 * c4 + 4 * wi;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f = hv ? bf2f(qrow[d0 + j]) * a.qscale : 0.f;
          f = __half2float(__float2half_rn(f));  // the value the MMA sees
          v[j] = f;
          s += f;
        }
        const int kb = 4 * g + wi;
        qa[kb][rr] = pack_h2(v[0], v[1]);      // reg0 (row r) / reg1 (row r+8): dims {0,1}
        qa[kb][2 + rr] = pack_h2(v[2], v[3]);  // reg2 / reg3: dims {2,3}
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      qsum[g][rr] = s;
    }
  }

  float m[2] = {-INFINITY, -INFINITY};  // running max per row (r, r+8), log2 domain
  float l[2] = {0.f, 0.f};              // thread-partial row sums
  float ob[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [group][row] bias term, thread-partial
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  uint16_t* vt = vtile[warp];
  const uint32_t vt_s = static_cast<uint32_t>(__cvta_generic_to_shared(vt));

  for (int t0 = k_begin + 16 * warp; t0 < k_end; t0 += 16 * QA_WARPS) {
    // ---- K fragments: key rows t0 + 8*nt + r, words 4c4.. (group 0) and 16+4c4.. (group 1)
    uint4 kw[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int row = min(t0 + 8 * nt + r, a.n - 1);
      const uint32_t* kr = a.kq + (head_row0 + row) * 32;
      kw[nt][0] = *reinterpret_cast<const uint4*>(kr + 4 * c4);
      kw[nt][1] = *reinterpret_cast<const uint4*>(kr + 16 + 4 * c4);
    }
    // scales/biases of the C-fragment keys t0 + 8nt + 2c4 + {0,1}: .x = key 0 {g0, g1},
    // .y = key 1 {g0, g1} (rows clamped to n - 1; those keys are masked below)
    uint2 ksc[2], kbi[2], vsc[2], vbi[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const size_t o0 = (head_row0 + min(t0 + 8 * nt + 2 * c4, a.n - 1)) * 2;
      const size_t o1 = (head_row0 + min(t0 + 8 * nt + 2 * c4 + 1, a.n - 1)) * 2;
      ksc[nt] = make_uint2(*reinterpret_cast<const uint32_t*>(a.ks + o0),
                           *reinterpret_cast<const uint32_t*>(a.ks + o1));
      kbi[nt] = make_uint2(*reinterpret_cast<const uint32_t*>(a.kb + o0),
                           *reinterpret_cast<const uint32_t*>(a.kb + o1));
      vsc[nt] = make_uint2(*reinterpret_cast<const uint32_t*>(a.vs + o0),
                           *reinterpret_cast<const uint32_t*>(a.vs + o1));
      vbi[nt] = make_uint2(*reinterpret_cast<const uint32_t*>(a.vb + o0),
                           *reinterpret_cast<const uint32_t*>(a.vb + o1));
    }
    // ---- V tile (16 keys x 128 codes) -> fp16 codes in swizzled shared memory ----
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = 4 * j + (lane >> 3);
      const int row = min(t0 + key, a.n - 1);
      const uint4 w = *reinterpret_cast<const uint4*>(a.vq + (head_row0 + row) * 32 + 4 * (lane & 7));
      uint4 lo, hi;
      lo.x = codes_h2(w.x, 0x4140u);
      lo.y = codes_h2(w.x, 0x4342u);
      lo.z = codes_h2(w.y, 0x4140u);
      lo.w = codes_h2(w.y, 0x4342u);
      hi.x = codes_h2(w.z, 0x4140u);
      hi.y = codes_h2(w.z, 0x4342u);
      hi.z = codes_h2(w.w, 0x4140u);
      hi.w = codes_h2(w.w, 0x4342u);
      const int ch = 2 * (lane & 7);
      *reinterpret_cast<uint4*>(vt + key * QA_D + ((ch ^ (key & 7)) * 8)) = lo;
      *reinterpret_cast<uint4*>(vt + key * QA_D + (((ch + 1) ^ (key & 7)) * 8)) = hi;
    }

    // ---- S = Q K^T per group, then the affine fold ----
    float sc[2][4];  // [n-tile][d0..d3]
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) {
        const uint4 kv = kw[nt][kb >> 2];
        const uint32_t w = (kb & 3) == 0 ? kv.x : (kb & 3) == 1 ? kv.y : (kb & 3) == 2 ? kv.z : kv.w;
        const uint32_t b0 = codes_h2(w, 0x4140u), b1 = codes_h2(w, 0x4342u);
        if (kb < 4)
          mma_f16(s0, qa[kb][0], qa[kb][1], qa[kb][2], qa[kb][3], b0, b1);
        else
          mma_f16(s1, qa[kb][0], qa[kb][1], qa[kb][2], qa[kb][3], b0, b1);
      }
      // keys t0 + 8nt + 2c4 + {0,1}; scales packed {k0g0, k0g1, k1g0, k1g1}
      const float ks00 = bfl(ksc[nt].x), ks01 = bfh(ksc[nt].x);
      const float ks10 = bfl(ksc[nt].y), ks11 = bfh(ksc[nt].y);
      const float kb00 = bfl(kbi[nt].x), kb01 = bfh(kbi[nt].x);
      const float kb10 = bfl(kbi[nt].y), kb11 = bfh(kbi[nt].y);
      const int key0 = t0 + 8 * nt + 2 * c4;
      const bool v0 = key0 < k_end, v1 = key0 + 1 < k_end;
      // rows r (d0, d1) and r + 8 (d2, d3)
      sc[nt][0] = v0 ? ks00 * s0[0] + ks01 * s1[0] + kb00 * qsum[0][0] + kb01 * qsum[1][0] : -INFINITY;
      sc[nt][1] = v1 ? ks10 * s0[1] + ks11 * s1[1] + kb10 * qsum[0][0] + kb11 * qsum[1][0] : -INFINITY;
      sc[nt][2] = v0 ? ks00 * s0[2] + ks01 * s1[2] + kb00 * qsum[0][1] + kb01 * qsum[1][1] : -INFINITY;
      sc[nt][3] = v1 ? ks10 * s0[3] + ks11 * s1[3] + kb10 * qsum[0][1] + kb11 * qsum[1][1] : -INFINITY;
    }

    // ---- online softmax (rows r and r+8) ----
    float corr[2], pv[2][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      float mx = fmaxf(fmaxf(sc[0][2 * rr], sc[0][2 * rr + 1]), fmaxf(sc[1][2 * rr], sc[1][2 * rr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[rr], mx);
      const float ref = (mn == -INFINITY) ? 0.f : mn;
      corr[rr] = exp2f(m[rr] - ref);
      m[rr] = mn;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pv[nt][2 * rr] = exp2f(sc[nt][2 * rr] - ref);
        pv[nt][2 * rr + 1] = exp2f(sc[nt][2 * rr + 1] - ref);
      }
      l[rr] = l[rr] * corr[rr] + pv[0][2 * rr] + pv[0][2 * rr + 1] + pv[1][2 * rr] + pv[1][2 * rr + 1];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      acc[i][0] *= corr[0];
      acc[i][1] *= corr[0];
      acc[i][2] *= corr[1];
      acc[i][3] *= corr[1];
    }
    // bias term and the P' = p * vs * 256 fragments per group
    uint32_t pa[2][4];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        float o = ob[g][rr] * corr[rr];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float vb0 = g ? bfh(vbi[nt].x) : bfl(vbi[nt].x);
          const float vb1 = g ? bfh(vbi[nt].y) : bfl(vbi[nt].y);
          o += pv[nt][2 * rr] * vb0 + pv[nt][2 * rr + 1] * vb1;
        }
        ob[g][rr] = o;
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float vs0 = (g ? bfh(vsc[nt].x) : bfl(vsc[nt].x)) * QA_PSCALE;
        const float vs1 = (g ? bfh(vsc[nt].y) : bfl(vsc[nt].y)) * QA_PSCALE;
        // A regs: reg0 row r keys 2c4.. (nt 0), reg1 row r+8 (nt 0), reg2 row r (nt 1), reg3 row r+8 (nt 1)
        pa[g][nt == 0 ? 0 : 2] = pack_h2(pv[nt][0] * vs0, pv[nt][1] * vs1);
        pa[g][nt == 0 ? 1 : 3] = pack_h2(pv[nt][2] * vs0, pv[nt][3] * vs1);
      }
    }
    __syncwarp();
    // ---- O += P' V (16 dim tiles of 8; tiles 0-7 group 0, 8-15 group 1) ----
#pragma unroll
    for (int dt = 0; dt < 16; dt += 2) {
      const int mtx = lane >> 3, rowm = lane & 7;
      const int key = (mtx & 1) * 8 + rowm;
      const int chunk = dt + (mtx >> 1);
      const uint32_t addr = vt_s + (uint32_t)(key * QA_D + ((chunk ^ (key & 7)) * 8)) * 2u;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_trans(addr, b0, b1, b2, b3);
      const int g = dt >> 3;
      mma_f16(acc[dt], pa[g][0], pa[g][1], pa[g][2], pa[g][3], b0, b1);
      mma_f16(acc[dt + 1], pa[g][0], pa[g][1], pa[g][2], pa[g][3], b2, b3);
    }
    __syncwarp();
  }

  // ---- reduce thread partials over the 4 lanes of a row, then merge the warps ----
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      ob[g][rr] += __shfl_xor_sync(0xffffffffu, ob[g][rr], 1);
      ob[g][rr] += __shfl_xor_sync(0xffffffffu, ob[g][rr], 2);
    }
  }
  if (c4 == 0) {
    s_m[warp][r] = m[0];
    s_m[warp][r + 8] = m[1];
    s_l[warp][r] = l[0];
    s_l[warp][r + 8] = l[1];
  }
  for (int i = threadIdx.x; i < 16 * (QA_D + 4); i += blockDim.x) (&s_acc[0][0])[i] = 0.f;
  __syncthreads();
  float wsc[2];  // this warp's weight in the CTA merge, per row
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int h = r + 8 * rr;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < QA_WARPS; ++w) mm = fmaxf(mm, s_m[w][h]);
    wsc[rr] = (m[rr] == -INFINITY) ? 0.f : exp2f(m[rr] - mm);
  }
  // accumulate this warp's scaled acc (+ bias term) into s_acc with shared atomics
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int g = dt >> 3;
    const int d = 8 * dt + 2 * c4;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int h = r + 8 * rr;
      const float o0 = acc[dt][2 * rr] * (1.0f / QA_PSCALE) + ob[g][rr];
      const float o1 = acc[dt][2 * rr + 1] * (1.0f / QA_PSCALE) + ob[g][rr];
      atomicAdd(&s_acc[h][d], o0 * wsc[rr]);
      atomicAdd(&s_acc[h][d + 1], o1 * wsc[rr]);
    }
  }
  __syncthreads();
  // write this CTA's partial: per head (M, L, acc[D])
  const size_t pbase = (((size_t)b * a.Hkv + hk) * a.nsplit + split) * (size_t)G * (QA_D + 2);
  for (int i = threadIdx.x; i < G * QA_D; i += blockDim.x) {
    const int h = i / QA_D, d = i % QA_D;
    a.part[pbase + (size_t)h * (QA_D + 2) + 2 + d] = s_acc[h][d];
  }
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float mm = -INFINITY, L = 0.f;
    for (int w = 0; w < QA_WARPS; ++w) mm = fmaxf(mm, s_m[w][h]);
    for (int w = 0; w < QA_WARPS; ++w)
      L += (s_m[w][h] == -INFINITY) ? 0.f : s_l[w][h] * exp2f(s_m[w][h] - mm);
    a.part[pbase + (size_t)h * (QA_D + 2) + 0] = mm;
    a.part[pbase + (size_t)h * (QA_D + 2) + 1] = L;
  }
  // ---- last CTA of this (batch, kv head) merges all splits ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.counters[b * a.Hkv + hk], 1);
    s_last = (prev == a.nsplit - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const size_t hbase = ((size_t)b * a.Hkv + hk) * a.nsplit * (size_t)G * (QA_D + 2);
  for (int i = threadIdx.x; i < G * (QA_D / 4); i += blockDim.x) {
    const int h = i / (QA_D / 4), d4 = (i % (QA_D / 4)) * 4;
    float mm = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s)
      mm = fmaxf(mm, __ldcg(a.part + hbase + ((size_t)s * G + h) * (QA_D + 2)));
    float L = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float* p = a.part + hbase + ((size_t)s * G + h) * (QA_D + 2);
      const float ms = __ldcg(p);
      if (ms == -INFINITY) continue;
      const float wv = exp2f(ms - mm);
      L += wv * __ldcg(p + 1);
      o0 += wv * __ldcg(p + 2 + d4);
      o1 += wv * __ldcg(p + 3 + d4);
      o2 += wv * __ldcg(p + 4 + d4);
      o3 += wv * __ldcg(p + 5 + d4);
    }
    const float inv = 1.0f / L;
    __nv_bfloat16* o = a.out + ((size_t)b * a.Hq + hk * G + h) * QA_D + d4;
    o[0] = __float2bfloat16_rn(o0 * inv);
    o[1] = __float2bfloat16_rn(o1 * inv);
    o[2] = __float2bfloat16_rn(o2 * inv);
    o[3] = __float2bfloat16_rn(o3 * inv);
  }
  if (threadIdx.x == 0) a.counters[b * a.Hkv + hk] = 0;  // leave the counter at zero
}

static void q8_split(int B, int Hkv, int n, int* kpc, int* nsplit) {
  const int target_ctas = 148 * 2;
  int per_head = (target_ctas + B * Hkv - 1) / (B * Hkv);
  if (per_head < 1) per_head = 1;
  int k = (n + per_head - 1) / per_head;
  k = (k + 63) / 64 * 64;
  if (k < 64) k = 64;
  *kpc = k;
  *nsplit = (n + k - 1) / k;
}

static size_t q8_ws(int B, int Hq, int Hkv, int n, size_t* counters_bytes) {
  int kpc, ns;
  q8_split(B, Hkv, n < 1 ? 1 : n, &kpc, &ns);
  const int G = Hq / (Hkv > 0 ? Hkv : 1);
  size_t cb = align_up(sizeof(int) * (size_t)B * Hkv, 256);
  if (counters_bytes) *counters_bytes = cb;
  return cb + align_up(sizeof(float) * (size_t)B * Hkv * ns * G * (QA_D + 2), 256);
}

int launch_q8_decode(const Q8Args& base, float scale, void* ws, size_t counters_bytes,
                     cudaStream_t st) {
  Q8Args a = base;
  q8_split(a.B, a.Hkv, a.n, &a.kpc, &a.nsplit);
  a.qscale = scale * 1.4426950408889634f;
  a.counters = static_cast<int*>(ws);
  a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + counters_bytes);
  dim3 grid(a.nsplit, a.Hkv, a.B);
  prof_begin("q8_decode", st);
  q8_decode_kernel<<<grid, QA_WARPS * 32, 0, st>>>(a);
  prof_end("q8_decode", st);
  LG_LAUNCH_CHECK("q8_decode");
  return LG_OK;
}

int check_q8_args(const void* q, int B, int Hq, int Hkv, int D, const uint32_t* k_q,
                  const void* k_s, const void* k_b, const uint32_t* v_q, const void* v_s,
                  const void* v_b, int cap, int n, void* out) {
  LG_CHECK_ARG(D == QA_D, "q8 decode: head_dim %d != 128 (decode only, head_dim 128)", D);
  LG_CHECK_ARG(B >= 1 && Hkv >= 1 && Hq >= 1 && Hq % Hkv == 0,
               "q8 decode: bad heads Hq=%d Hkv=%d B=%d", Hq, Hkv, B);
  LG_CHECK_ARG(Hq / Hkv <= 16, "q8 decode: %d q heads per kv head is too many (max 16)",
               Hq / Hkv);
  LG_CHECK_ARG(n >= 1 && n <= cap, "q8 decode: need 1 <= n (%d) <= cap (%d)", n, cap);
  LG_CHECK_ARG(q && k_q && k_s && k_b && v_q && v_s && v_b && out, "q8 decode: NULL pointer");
  LG_CHECK_ARG(aligned(k_q, 16) && aligned(v_q, 16) && aligned(k_s, 4) && aligned(k_b, 4) &&
                   aligned(v_s, 4) && aligned(v_b, 4),
               "q8 decode: packed K/V must be 16-byte aligned, scales/biases 4-byte aligned");
  return LG_OK;
}

}  // namespace lg

using namespace lg;

extern "C" size_t lg_q8_decode_workspace_bytes(int B, int Hq, int Hkv, int n) {
  if (B < 1 || Hkv < 1 || Hq < Hkv) return 0;
  return q8_ws(B, Hq, Hkv, n, nullptr);
}

extern "C" int lg_q8_decode_attention(const void* q, int B, int Hq, int Hkv, int D,
                                      const uint32_t* k_q, const void* k_s, const void* k_b,
                                      const uint32_t* v_q, const void* v_s, const void* v_b,
                                      int cap, int n, float scale, void* out, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  int rc = check_q8_args(q, B, Hq, Hkv, D, k_q, k_s, k_b, v_q, v_s, v_b, cap, n, out);
  if (rc) return rc;
  size_t cb;
  const size_t need = q8_ws(B, Hq, Hkv, n, &cb);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "q8 decode: workspace %zu bytes at %p, need %zu (256-aligned)",
                workspace_bytes, workspace, need);
  Q8Args a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kq = k_q;
  a.ks = static_cast<const __nv_bfloat16*>(k_s);
  a.kb = static_cast<const __nv_bfloat16*>(k_b);
  a.vq = v_q;
  a.vs = static_cast<const __nv_bfloat16*>(v_s);
  a.vb = static_cast<const __nv_bfloat16*>(v_b);
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.cap = cap;
  a.n = n;
  a.out = static_cast<__nv_bfloat16*>(out);
  return launch_q8_decode(a, scale, workspace, cb, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
// Fixed-scratch variant: the same kernel with its split partials and completion counters in
// a file-scope device array instead of a caller workspace, for callers that cannot allocate
// device memory when they call. The array's device address is looked up once per device
// with cudaGetSymbolAddress (in host code the symbol name is only a stand-in).
// ---------------------------------------------------------------------------------------
#include <mutex>

namespace lg {

constexpr size_t Q8_FIXED_SCRATCH_BYTES = (size_t)4 << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char q8_fixed_scratch[Q8_FIXED_SCRATCH_BYTES];

constexpr int Q8_MAX_DEVICES = 64;
static std::mutex q8_fixed_mu;
static void* q8_fixed_ptr[Q8_MAX_DEVICES] = {};

static int q8_fixed_base(void** out) {
  int dev = 0;
  LG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= Q8_MAX_DEVICES)
    return fail(LG_ERR_UNSUPPORTED, "q8 decode (fixed scratch): device %d out of range", dev);
  std::lock_guard<std::mutex> lock(q8_fixed_mu);
  if (!q8_fixed_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, q8_fixed_scratch);
    if (e != cudaSuccess || !p)
      return fail(LG_ERR_CUDA, "q8 decode (fixed scratch): cudaGetSymbolAddress: %s",
                  cudaGetErrorString(e));
    q8_fixed_ptr[dev] = p;
  }
  *out = q8_fixed_ptr[dev];
  return LG_OK;
}

}  // namespace lg

extern "C" size_t lg_q8_decode_fixed_scratch_bytes(void) { return lg::Q8_FIXED_SCRATCH_BYTES; }

extern "C" int lg_q8_decode_attention_noalloc(const void* q, int B, int Hq, int Hkv, int D,
                                              const uint32_t* k_q, const void* k_s,
                                              const void* k_b, const uint32_t* v_q,
                                              const void* v_s, const void* v_b, int cap, int n,
                                              float scale, void* out, void* stream) {
  int rc = check_q8_args(q, B, Hq, Hkv, D, k_q, k_s, k_b, v_q, v_s, v_b, cap, n, out);
  if (rc) return rc;
  size_t cb;
  const size_t need = q8_ws(B, Hq, Hkv, n, &cb);
  if (need > Q8_FIXED_SCRATCH_BYTES)
    return fail(LG_ERR_INVALID,
                "q8 decode (fixed scratch): this call needs %zu bytes of scratch, more than the "
                "fixed %zu (use lg_q8_decode_attention with a caller workspace)",
                need, Q8_FIXED_SCRATCH_BYTES);
  void* base = nullptr;
  rc = q8_fixed_base(&base);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the completion counters must start at zero; a completed call leaves them at zero, but a
  // call that was cut short would not, so clear them on every call
  LG_CUDA_TRY(cudaMemsetAsync(base, 0, cb, st));
  Q8Args a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kq = k_q;
  a.ks = static_cast<const __nv_bfloat16*>(k_s);
  a.kb = static_cast<const __nv_bfloat16*>(k_b);
  a.vq = v_q;
  a.vs = static_cast<const __nv_bfloat16*>(v_s);
  a.vb = static_cast<const __nv_bfloat16*>(v_b);
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.cap = cap;
  a.n = n;
  a.out = static_cast<__nv_bfloat16*>(out);
  return launch_q8_decode(a, scale, base, cb, st);
}
