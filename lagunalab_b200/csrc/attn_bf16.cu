// Single-token attention over a bf16 KV cache (laguna_mlx/laguna.py:99-107, the SDPA branch
// of Attention.__call__ with KVCache), split over the keys: softmax(q . K[:n]^T * scale) . V[:n]
// per query head, GQA group up to 16, head_dim 128.
//
// Grid (splits, kv heads, batch); each CTA (4 warps) owns a contiguous range of 16-key tiles
// of one kv head; each warp walks every 4th tile with a one-tile register prefetch. Both
// products run on mma.sync m16n8k16 (bf16 in, fp32 accumulate):
//   S^T = K Q^T   (M = 16 keys, N = 8 query heads, K = 16 dims): a GQA group of 8 fills N;
//   O^T = V^T P^T (M = 16 dims, N = heads, K = 16 keys).
// Lane (r, c4) loads, for keys r and r + 8 of a tile, the 16-byte pieces at dims
// 32j + 8c4 .. +7 (j = 0..3) of both K and V rows (each row read in 64-byte runs by 4 lanes).
// For S^T the contraction order inside a 16-wide k-block is permuted to match those pieces
// (q uses the same order). For O^T, movmatrix transposes 8x8 blocks of the V pieces in
// registers into the V^T operand, so V never goes through shared memory. q enters unscaled
// (it is already bf16); scale * log2(e) is applied to the fp32 scores. P is rounded to bf16
// for the MMA. The number of valid keys can come from a device counter (decode steps driven
// without the host); the output gate of laguna.py:105-106 is applied in the final write:
// out = bf16(bf16(o) * gate).
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace lg {

constexpr int AB_D = 128;
constexpr int AB_WARPS = 4;
constexpr int AB_THREADS = AB_WARPS * 32;
constexpr int AB_TK = 16;  // keys per tile
constexpr size_t AB_CTRL_BYTES = 16384;  // completion counters, one 128-byte slot per (b, kv head)
constexpr int AB_CTRL_SLOTS = (int)(AB_CTRL_BYTES / 128);
constexpr int AB_MERGE_MAX = AB_WARPS * 16 * (AB_D + 1);  // split x head weights in the slab
constexpr int AB_MIN_WARP_TILES = 4;  // plan at least this many 16-key tiles per warp

__device__ __forceinline__ void mma_bf16_ab(float (&d)[4], uint32_t a0, uint32_t a1,
                                            uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  __syncwarp();  // mma.sync.aligned needs the whole warp converged
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movtrans_ab(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float ex2_ab(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct AbArgs {
  const __nv_bfloat16* q;   // [B, Hq, D]
  const __nv_bfloat16* k;   // [B, Hkv, cap, D]
  const __nv_bfloat16* v;
  const __nv_bfloat16* gate;  // [B, Hq] per-head output gate, or null
  const int* n_dev;         // valid keys = n_dev[b * n_stride] + n_add when non-null, else n_host
  int n_host, n_add;
  int n_stride;             // 0: one length for every batch row; 1: per stream (batched decode)
  int B, Hq, Hkv, G, cap, tpc, nsplit;
  float qscale;             // scale * log2(e)
  int* counters;            // [B * Hkv][32] (nsplit > 1); bit 20 and up: unused here
  float2* part_ml;          // [B * Hkv][nsplit][G]
  float* part_acc;          // [B * Hkv][nsplit][G][D]
  __nv_bfloat16* out;       // [B, Hq, D]
};

template <int NT>
__global__ void __launch_bounds__(AB_THREADS) bf16_decode_kernel(const AbArgs a) {
  __shared__ float slab[AB_WARPS][16][AB_D + 1];
  __shared__ float s_m[AB_WARPS][16], s_l[AB_WARPS][16], s_wt[AB_WARPS][16];
  __shared__ float s_M[16], s_L[16];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c4 = lane & 3;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G;
  const int bh = b * a.Hkv + hk;
  int n = a.n_dev ? a.n_dev[b * a.n_stride] + a.n_add : a.n_host;
  // the row the previous kernel appends: n - 1, or, in a sliding window's ring buffer that
  // has wrapped (n > cap), position n - 1 mod cap
  const int newest = n > a.cap ? (n - 1) % a.cap : n - 1;
  n = min(max(n, 0), a.cap);
  const int tile_lo = split * a.tpc;
  const int tile_hi = min(tile_lo + a.tpc, (n + AB_TK - 1) / AB_TK);
  const __nv_bfloat16* kbase = a.k + (size_t)bh * a.cap * AB_D;
  const __nv_bfloat16* vbase = a.v + (size_t)bh * a.cap * AB_D;

  float m[NT][2], l[NT][2], acc[NT][8][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[nt][i][0] = acc[nt][i][1] = acc[nt][i][2] = acc[nt][i][3] = 0.f;
  }

  auto load_tile = [&](int tile, uint4 (&kw)[2][4], uint4 (&vw)[2][4]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int key = min(tile * AB_TK + r + 8 * i, n - 1);
      const __nv_bfloat16* kr = kbase + (size_t)key * AB_D + 8 * c4;
      const __nv_bfloat16* vr = vbase + (size_t)key * AB_D + 8 * c4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kw[i][j] = ldg_stream_u4(kr + 32 * j);
        vw[i][j] = ldg_stream_u4(vr + 32 * j);
      }
    }
  };

  // Before the PDL wait: the length comes from a counter the previous kernel does not write,
  // and the first tile is loaded unless it holds the newest row (the previous kernel appends
  // it); everything else (q, the newest row, the gate) is read after the wait.
  uint4 kw[2][4], vw[2][4], kn[2][4], vn[2][4];
  int tile = tile_lo + warp;
  const bool early = tile < tile_hi && (newest < tile * AB_TK || newest >= tile * AB_TK + AB_TK);
  if (early) load_tile(tile, kw, vw);
  pdl_wait();
  pdl_trigger();
  if (tile < tile_hi && !early) load_tile(tile, kw, vw);
  // Q^T fragments: k-block kb = 2j + e, b0 = dims 32j + 8c4 + 4e + {0,1}, b1 = + {2,3}
  uint32_t qb[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = r + 8 * nt;
    const bool hv = h < G;
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        a.q + ((size_t)b * a.Hq + hk * G + (hv ? h : 0)) * AB_D);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = hv ? *reinterpret_cast<const uint4*>(qrow + 16 * j + 4 * c4)
                         : make_uint4(0, 0, 0, 0);
      qb[nt][2 * j][0] = w.x;
      qb[nt][2 * j][1] = w.y;
      qb[nt][2 * j + 1][0] = w.z;
      qb[nt][2 * j + 1][1] = w.w;
    }
  }


  for (; tile < tile_hi; tile += AB_WARPS) {
    const int next = tile + AB_WARPS;
    if (next < tile_hi) load_tile(next, kn, vn);
    // ---- S^T = K Q^T ----
    float sa[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sa[nt][0] = sa[nt][1] = sa[nt][2] = sa[nt][3] = 0.f;
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
      const int j = kb >> 1, e = kb & 1;
      const uint32_t a0 = u4w(kw[0][j], 2 * e), a2 = u4w(kw[0][j], 2 * e + 1);
      const uint32_t a1 = u4w(kw[1][j], 2 * e), a3 = u4w(kw[1][j], 2 * e + 1);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_bf16_ab(sa[nt], a0, a1, a2, a3, qb[nt][kb][0], qb[nt][kb][1]);
    }
    const int t0 = tile * AB_TK;
    const bool v0 = t0 + r < n, v1 = t0 + r + 8 < n;
    float p[NT][2][2], corr[NT][2];
    bool rescale = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float s0 = v0 ? sa[nt][hh] * a.qscale : -INFINITY;
        const float s1 = v1 ? sa[nt][2 + hh] * a.qscale : -INFINITY;
        float mx = fmaxf(s0, s1);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[nt][hh], mx);
        const float ref = (mn == -INFINITY) ? 0.f : mn;
        const float cr = ex2_ab(m[nt][hh] - ref);
        rescale |= (cr != 1.f);
        corr[nt][hh] = cr;
        m[nt][hh] = mn;
        p[nt][0][hh] = ex2_ab(s0 - ref);
        p[nt][1][hh] = ex2_ab(s1 - ref);
        l[nt][hh] = l[nt][hh] * cr + p[nt][0][hh] + p[nt][1][hh];
      }
    }
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[nt][i][0] *= corr[nt][0];
          acc[nt][i][1] *= corr[nt][1];
          acc[nt][i][2] *= corr[nt][0];
          acc[nt][i][3] *= corr[nt][1];
        }
    }
    // ---- P^T into the B layout; V^T fragments by transposing the V pieces ----
    uint32_t bp[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      bp[nt][0] = movtrans_ab(pack_bf2(p[nt][0][0], p[nt][0][1]));
      bp[nt][1] = movtrans_ab(pack_bf2(p[nt][1][0], p[nt][1][1]));
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {  // rows r: dim 32j + 8(r/2) + 2i + r%2, rows r+8: i + 1
      const int j = mt >> 1, i = 2 * (mt & 1);
      const uint32_t a0 = movtrans_ab(u4w(vw[0][j], i)), a1 = movtrans_ab(u4w(vw[0][j], i + 1));
      const uint32_t a2 = movtrans_ab(u4w(vw[1][j], i)), a3 = movtrans_ab(u4w(vw[1][j], i + 1));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_bf16_ab(acc[nt][mt], a0, a1, a2, a3, bp[nt][0], bp[nt][1]);
    }
    if (next < tile_hi) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          kw[i][j] = kn[i][j];
          vw[i][j] = vn[i][j];
        }
    }
  }

  // ---- merge the warps of this CTA ----
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) l[nt][hh] += __shfl_xor_sync(0xffffffffu, l[nt][hh], o);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int head = 2 * c4 + hh + 8 * nt;
      if (head < G) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int j = mt >> 1, i = 2 * (mt & 1);
          slab[warp][head][32 * j + 8 * (r >> 1) + 2 * i + (r & 1)] = acc[nt][mt][hh];
          slab[warp][head][32 * j + 8 * (r >> 1) + 2 * (i + 1) + (r & 1)] = acc[nt][mt][2 + hh];
        }
        if (r == 0) {
          s_m[warp][head] = m[nt][hh];
          s_l[warp][head] = l[nt][hh];
        }
      }
    }
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < AB_WARPS; ++w) M = fmaxf(M, s_m[w][h]);
    float L = 0.f;
    for (int w = 0; w < AB_WARPS; ++w) {
      const float wt = (s_m[w][h] == -INFINITY) ? 0.f : ex2_ab(s_m[w][h] - M);
      s_wt[w][h] = wt;
      L += wt * s_l[w][h];
    }
    s_M[h] = M;
    s_L[h] = L;
  }
  __syncthreads();
  const int ns = a.nsplit;
  if (ns == 1) {  // whole (batch, kv head) in this CTA: normalise, gate, write
    for (int i = threadIdx.x; i < G * AB_D; i += AB_THREADS) {
      const int h = i / AB_D, d = i % AB_D;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < AB_WARPS; ++w) v += s_wt[w][h] * slab[w][h][d];
      float o = round_bf16(v / s_L[h]);
      if (a.gate) o *= bf2f(a.gate[(size_t)b * a.Hq + hk * G + h]);
      a.out[((size_t)b * a.Hq + hk * G + h) * AB_D + d] = __float2bfloat16_rn(o);
    }
    return;
  }
  const size_t pbase = ((size_t)bh * ns + split) * G;
  for (int i = threadIdx.x; i < G * AB_D; i += AB_THREADS) {
    const int h = i / AB_D, d = i % AB_D;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < AB_WARPS; ++w) v += s_wt[w][h] * slab[w][h][d];
    a.part_acc[(pbase + h) * AB_D + d] = v;
  }
  if (threadIdx.x < G) a.part_ml[pbase + threadIdx.x] = make_float2(s_M[threadIdx.x], s_L[threadIdx.x]);
  __syncthreads();  // this split's partials are stored before thread 0 releases them
  int* ctr = a.counters + bh * 32;
  if (threadIdx.x == 0) s_last = (atom_add_acq_rel_gpu(ctr, 1) == ns - 1);
  __syncthreads();  // the merger: every split's partials, acquired by thread 0, are visible
  if (!s_last) return;
  // ---- the last CTA of this (batch, kv head) merges the splits: split weights staged in
  // shared memory (reusing the slab), then each thread sums its float4 items over the
  // splits with 16 loads in flight ----
  const size_t hbase = (size_t)bh * ns * G;
  float* t_w = &slab[0][0][0];  // [split][G] normalised weights (ns * G <= AB_MERGE_MAX)
  for (int i = threadIdx.x; i < ns * G; i += AB_THREADS) t_w[i] = __ldcg(&a.part_ml[hbase + i].x);
  __syncthreads();
  for (int h = warp; h < G; h += AB_WARPS) {  // one warp per head
    float M = -INFINITY;
    for (int s = lane; s < ns; s += 32) M = fmaxf(M, t_w[s * G + h]);
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < ns; s += 32) {
      const float mx = t_w[s * G + h];
      const float w = (mx == -INFINITY) ? 0.f : ex2_ab(mx - M);
      L += w * __ldcg(&a.part_ml[hbase + (size_t)s * G + h].y);
      t_w[s * G + h] = w;
    }
    L = warp_sum(L);
    if (lane == 0) s_L[h] = 1.f / L;
  }
  __syncthreads();
  const float4* pacc = reinterpret_cast<const float4*>(a.part_acc) + hbase * (AB_D / 4);
  for (int it = threadIdx.x; it < G * (AB_D / 4); it += AB_THREADS) {
    const int h = it / (AB_D / 4), d4 = it % (AB_D / 4);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < ns; s0 += 16) {
      float4 vv[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        if (s0 + u < ns) vv[u] = __ldcg(pacc + ((size_t)(s0 + u) * G + h) * (AB_D / 4) + d4);
#pragma unroll
      for (int u = 0; u < 16; ++u)
        if (s0 + u < ns) {
          const float w = t_w[(s0 + u) * G + h];
          o.x += w * vv[u].x;
          o.y += w * vv[u].y;
          o.z += w * vv[u].z;
          o.w += w * vv[u].w;
        }
    }
    const float il = s_L[h];
    const float gt = a.gate ? bf2f(a.gate[(size_t)b * a.Hq + hk * G + h]) : 1.f;
    const float ov[4] = {o.x, o.y, o.z, o.w};
    __nv_bfloat16* dst = a.out + ((size_t)b * a.Hq + hk * G + h) * AB_D + 4 * d4;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float y = round_bf16(ov[c] * il);
      if (a.gate) y *= gt;
      dst[c] = __float2bfloat16_rn(y);
    }
  }
  if (threadIdx.x == 0) ctr[0] = 0;  // leave the counter at zero for the next call
}

static int ab_sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return 148;
  }
  if (!cached[dev]) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) {
      (void)cudaGetLastError();
      c = 148;
    }
    cached[dev] = c;
  }
  return cached[dev];
}

// splits per (batch, kv head) for a planned length: about two CTAs per SM in total, at least
// four tiles per warp (shorter splits spend more on the merge than they save); one split when
// B * Hkv is large (no merge, no counters).
static void ab_split(int B, int Hkv, int n_plan, int* tpc, int* nsplit) {
  const int BH = B * Hkv;
  const int tiles = (n_plan + AB_TK - 1) / AB_TK;
  int ns = (2 * ab_sm_count()) / BH;
  ns = min(ns, (tiles + AB_WARPS * AB_MIN_WARP_TILES - 1) / (AB_WARPS * AB_MIN_WARP_TILES));
  if (BH > AB_CTRL_SLOTS) ns = 1;
  ns = max(1, min(ns, 296));
  const int G = 16;  // worst case for the merge's weight table
  ns = min(ns, AB_MERGE_MAX / G);
  const int t = max(1, (tiles + ns - 1) / ns);
  *tpc = t;
  *nsplit = max(1, (tiles + t - 1) / t);
}

static size_t ab_ws(int B, int Hq, int Hkv, int n_plan, size_t* ml_off, size_t* acc_off) {
  int tpc, ns;
  ab_split(B, Hkv, n_plan < 1 ? 1 : n_plan, &tpc, &ns);
  const size_t G = (size_t)Hq / (Hkv > 0 ? Hkv : 1);
  const size_t parts = (size_t)B * Hkv * ns * G;
  const size_t ml = AB_CTRL_BYTES;
  const size_t acc = ml + (ns > 1 ? align_up(sizeof(float2) * parts, 256) : 0);
  if (ml_off) *ml_off = ml;
  if (acc_off) *acc_off = acc;
  return acc + (ns > 1 ? align_up(sizeof(float) * parts * AB_D, 256) : 0);
}

}  // namespace lg

using namespace lg;

extern "C" size_t lg_bf16_decode_workspace_bytes(int B, int Hq, int Hkv, int n_plan) {
  if (B < 1 || Hkv < 1 || Hq < Hkv) return 0;
  return ab_ws(B, Hq, Hkv, n_plan, nullptr, nullptr);
}

static int bf16_decode_run(const void* q, int B, int Hq, int Hkv, int D, const void* k,
                           const void* v, int cap, int n, const int32_t* n_dev, int n_stride,
                           int n_add, int n_plan, float scale, const void* gate, void* out,
                           void* workspace, size_t workspace_bytes, void* stream) {
  LG_CHECK_ARG(D == AB_D, "bf16 decode: head_dim %d != 128", D);
  LG_CHECK_ARG(B >= 1 && Hkv >= 1 && Hq >= 1 && Hq % Hkv == 0 && Hq / Hkv <= 16,
               "bf16 decode: bad heads Hq=%d Hkv=%d (group <= 16)", Hq, Hkv);
  LG_CHECK_ARG(cap >= 1 && (n_dev || (n >= 1 && n <= cap)),
               "bf16 decode: need 1 <= n (%d) <= cap (%d)", n, cap);
  LG_CHECK_ARG(n_plan >= 1 && n_plan <= cap, "bf16 decode: planned length %d not in [1, cap=%d]",
               n_plan, cap);
  LG_CHECK_ARG(q && k && v && out, "bf16 decode: NULL pointer");
  LG_CHECK_ARG(aligned(q, 16) && aligned(k, 16) && aligned(v, 16),
               "bf16 decode: q, K and V must be 16-byte aligned");
  size_t ml_off, acc_off;
  const size_t need = ab_ws(B, Hq, Hkv, n_plan, &ml_off, &acc_off);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "bf16 decode: workspace %zu bytes at %p, need %zu (256-aligned)",
                workspace_bytes, workspace, need);
  AbArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.n_dev = n_dev;
  a.n_host = n;
  a.n_add = n_add;
  a.n_stride = n_stride;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.cap = cap;
  ab_split(B, Hkv, n_plan, &a.tpc, &a.nsplit);
  a.qscale = scale * 1.4426950408889634f;
  char* base = static_cast<char*>(workspace);
  a.counters = reinterpret_cast<int*>(base);
  a.part_ml = reinterpret_cast<float2*>(base + ml_off);
  a.part_acc = reinterpret_cast<float*>(base + acc_off);
  a.out = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(a.nsplit, Hkv, B);
  prof_begin("bf16_decode", st);
  if (a.G <= 8)
    LG_CUDA_TRY(launch_k(bf16_decode_kernel<1>, grid, dim3(AB_THREADS), 0, st, a));
  else
    LG_CUDA_TRY(launch_k(bf16_decode_kernel<2>, grid, dim3(AB_THREADS), 0, st, a));
  prof_end("bf16_decode", st);
  LG_LAUNCH_CHECK("bf16_decode");
  return LG_OK;
}

extern "C" int lg_bf16_decode_attention(const void* q, int B, int Hq, int Hkv, int D,
                                        const void* k, const void* v, int cap, int n,
                                        const int32_t* n_dev, int n_add, int n_plan, float scale,
                                        const void* gate, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return bf16_decode_run(q, B, Hq, Hkv, D, k, v, cap, n, n_dev, 0, n_add, n_plan, scale, gate,
                         out, workspace, workspace_bytes, stream);
}

extern "C" int lg_bf16_decode_attention_streams(const void* q, int B, int Hq, int Hkv, int D,
                                                const void* k, const void* v, int cap,
                                                const int32_t* n_dev, int n_add, int n_plan,
                                                float scale, const void* gate, void* out,
                                                void* workspace, size_t workspace_bytes,
                                                void* stream) {
  LG_CHECK_ARG(n_dev, "bf16 decode streams: NULL lengths");
  return bf16_decode_run(q, B, Hq, Hkv, D, k, v, cap, 0, n_dev, 1, n_add, n_plan, scale, gate,
                         out, workspace, workspace_bytes, stream);
}
