// Fused split-KV decode attention over an MLX 8-bit group-64 KV cache
// (laguna_mlx/q8_attn.py:17-130), rebuilt for B200.
//
// Work split: grid (splits, kv heads, batch); each CTA owns a contiguous key range of one kv
// head and its whole GQA group (up to 16 query heads). Its 8 warps walk interleaved 32-key
// tiles; each warp streams its own tiles through a 3-stage ring in shared memory with TMA
// (packed K and V rows with the 128-byte swizzle, the four scale/bias arrays as 128-byte
// boxes). A warp first reads a whole stage into registers and refills it at once, so while
// it computes on one tile the next three are in flight; the two 16-key halves of a tile are
// independent MMA chains that share one online-softmax step. The CTA
// merges its warps, writes one partial per head, and the last CTA of each (batch, kv head) to
// finish merges the partials (the log-sum-exp merge of q8_attn.py:127-130) and writes the
// bf16 output, all in one launch. Completion is counted with one atomic per CTA; nothing
// waits on another CTA.
//
// Arithmetic: both products run on the tensor cores (mma.sync m16n8k16, fp16 in, fp32
// accumulate) on the raw 8-bit codes. The affine dequantisation value = scale * code + bias
// (q8_attn.py:50, :55) is folded in instead of applied per element:
//   score(t, h) = sum_g ks[t,g] * (q_h . code_k[t,g]) + kb[t,g] * sum(q_h[g])
//   out(d, h)   = sum_t (p[t,h] * vs[t,g(d)]) * code_v[t,d] + sum_t p[t,h] * vb[t,g(d)]
// A code c enters the MMA as the fp16 number 1024 + c (bit pattern 0x6400 | c: one byte
// permute, no subtraction). The 1024 offsets are removed exactly: for K through the bias
// term (kb - 1024 ks), for V by a second MMA of the same P' fragments against a matrix of
// ones (sum_t P'), subtracted at the end. Scores stay in the log2 domain (q pre-scaled by
// scale * log2 e); softmax, partials and the merge are fp32.
//
// Fragment layout. Scores are computed transposed, S^T = K Q^T (M = 16 keys, N = 8 query
// heads, K = 16 dims), so a GQA group of 8 fills the MMA's N exactly (16 heads: two N tiles).
// Query heads are the N columns of the output as well: O^T = V^T P'^T (M = 16 dims,
// N = heads, K = 16 keys); the P' fragment is moved from S^T's accumulator layout to the B
// operand layout with movmatrix. Within a 16-key tile, MMA row m is key kperm(m) (m < 8,
// +8 for m >= 8), kperm = 0 4 2 6 5 1 7 3: with the 128-byte swizzle this makes the K reads
// (16-byte) and the V reads (8-byte) free of shared-memory bank conflicts. Head-dim
// permutations inside a group are free (the contraction order does not matter and the
// output columns are written back in place).
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace lg {

using namespace tc;

constexpr int QA_D = 128;
constexpr int QA_WARPS = 8;
constexpr int QA_THREADS = QA_WARPS * 32;
constexpr int QA_STAGES = 3;
constexpr int QA_TK = 32;                              // keys per warp tile (two MMA halves)
constexpr int QA_TILE = QA_TK * 128;                   // bytes of one packed K (or V) tile
constexpr int QA_SC = QA_TK * 4;                       // bytes of one scale array per tile
constexpr int QA_SCS = QA_SC;  // their spacing in shared memory (tiled TMA: 128-byte aligned)
static_assert(QA_SCS % 128 == 0, "TMA destinations must be 128-byte aligned");
constexpr float QA_PSCALE = 256.0f;                    // keeps p * vs in fp16's normal range
constexpr int QA_MAX_SPLITS = 256;

// shared memory (offsets from a 1024-byte aligned base)
constexpr int QA_OFF_KV = 0;                                            // [warp][stage][K|V]
constexpr int QA_OFF_SC = QA_OFF_KV + QA_WARPS * QA_STAGES * 2 * QA_TILE;  // [warp][stage][4][128]
constexpr int QA_OFF_BAR = QA_OFF_SC + QA_WARPS * QA_STAGES * 4 * QA_SCS;  // [warp][stage]
constexpr int QA_OFF_ML = QA_OFF_BAR + QA_WARPS * QA_STAGES * 8;          // m, l, wt [warp][16]
constexpr int QA_OFF_HEAD = QA_OFF_ML + 3 * QA_WARPS * 16 * 4;            // M, L [16]
constexpr int QA_OFF_MBAR = QA_OFF_HEAD + 2 * 16 * 4;                     // merge mbarrier
constexpr int QA_OFF_FLAG = QA_OFF_MBAR + 8;                              // err, last
constexpr int QA_SMEM = QA_OFF_FLAG + 16 + 1024;                          // + alignment slack
// after the key loop the ring is reused: per-warp outputs, then the split merge tables
constexpr int QA_OFF_SLAB = 0;                                    // [warp][16][QA_SLAB] fp32
constexpr int QA_SLAB = QA_D + 1;  // padded row: the fragment stores of a warp spread over banks
// final merge: split partials [split][G][D] fp32, then (max, sum) [split][G], weights
// [split][G]; copied in whole when split x G <= QA_MERGE_SMEM, else read in batches
constexpr int QA_MERGE_SMEM = 368;
static_assert(QA_MERGE_SMEM * (QA_D * 4 + 8 + 4) + 32 <= QA_OFF_SC, "merge copy exceeds the ring");
static_assert(QA_MAX_SPLITS * 16 * (8 + 4) + 32 <= QA_OFF_SC, "merge tables exceed the ring");
static_assert(QA_WARPS * 16 * QA_SLAB * 4 <= QA_OFF_SC, "warp outputs exceed the ring");

// float2 (max, sum) entries per (batch, kv head), padded to 16 bytes for the bulk copy
__host__ __device__ constexpr int q8_ml_stride(int ns, int G) { return (ns * G + 1) & ~1; }

__device__ __forceinline__ uint32_t prmt32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// fp16x2 {1024 + byte i0, 1024 + byte i1} of a word (sel 0x4140: bytes 0, 1; 0x4342: 2, 3).
__device__ __forceinline__ uint32_t code_h2(uint32_t w, uint32_t sel) {
  return prmt32(w, 0x64646464u, sel);
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

// Transpose of an 8x8 16-bit matrix held in the MMA accumulator/operand fragment layout.
__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// 2^x (PTX ex2.approx: relative error ~2^-22; -inf -> 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float bfl(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bfh(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// key row of MMA row m (0..7) inside an 8-key half tile
__device__ __forceinline__ int kperm(int m) { return (0x37156240 >> (4 * m)) & 7; }

// byte offset of 16-byte chunk `chunk` of key row `key` in a 128-byte-swizzled tile
__device__ __forceinline__ int sw128(int key, int chunk) {
  return key * 128 + ((chunk ^ (key & 7)) << 4);
}

__device__ __forceinline__ uint32_t u4get(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct Q8Maps {
  CUtensorMap k, v;  // packed K / V rows: 32 words x 16 keys, 128-byte swizzle
  CUtensorMap s[4];  // ks, kb, vs, vb: 4 keys per 16-byte row, box 4 rows (16 keys)
};

struct Q8Args {
  const __nv_bfloat16* q;   // [B, Hq, D]
  const uint32_t* sc[4];    // ks, kb, vs, vb as one 32-bit word {g0, g1} per key
  int B, Hq, Hkv, G, cap, n;
  int tpc;                  // 32-key tiles per CTA (a contiguous range)
  int nsplit;               // CTAs per (batch, kv head)
  int zero;                 // always 0 (a value the compiler cannot fold)
  float qscale;             // scale * log2(e)
  int* counters;            // [B * Hkv][32]: finished CTAs per (batch, kv head) in word 0 of
                            // its 128-byte slot; bit 20 and up: a wait gave up (nsplit > 1)
  float2* part_ml;          // [B * Hkv][q8_ml_stride]: (max, sum) per split and head
  float* part_acc;          // [B * Hkv, nsplit, G, D]
  __nv_bfloat16* out;       // [B, Hq, D]
  const int* n_dev;         // the valid length is *n_dev + n_add (<= n, the planned length)
  int n_add;
  const __nv_bfloat16* gate;  // [B, Hq] per-head output gate, or null
  int early;                  // stream K/V tiles before the PDL wait (device-length calls)
};

// bf16(bf16(v) * gate) (the attention output times the per-head gate, laguna.py:105-106)
__device__ __forceinline__ float q8_gated(float v, const Q8Args& a, size_t head) {
  return a.gate ? round_bf16(v) * bf2f(a.gate[head]) : v;
}

template <int NT, bool SC_TMA>
__global__ void __launch_bounds__(QA_THREADS, 1)
    q8_decode_kernel(const __grid_constant__ Q8Maps mp, const Q8Args a) {
  extern __shared__ uint8_t q8_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(q8_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c4 = lane & 3;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G;
  const int bh = b * a.Hkv + hk;
  const int head_row0 = bh * a.cap;  // < 2^31 (checked on the host)
  const int tile0 = split * a.tpc;     // this CTA's tiles: [tile0, tile0 + tpc) of the head
  const int n_valid = a.n_dev ? min(*a.n_dev + a.n_add, a.n) : a.n;
  const int k_end = n_valid;

  uint8_t* kvw = sm + QA_OFF_KV + warp * QA_STAGES * 2 * QA_TILE;
  uint8_t* scw = sm + QA_OFF_SC + warp * QA_STAGES * 4 * QA_SCS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + QA_OFF_BAR) + warp * QA_STAGES;
  float* s_m = reinterpret_cast<float*>(sm + QA_OFF_ML);  // [warp][16]
  float* s_l = s_m + QA_WARPS * 16;
  float* s_wt = s_l + QA_WARPS * 16;
  float* s_M = reinterpret_cast<float*>(sm + QA_OFF_HEAD);
  float* s_L = s_M + 16;
  int* s_flag = reinterpret_cast<int*>(sm + QA_OFF_FLAG);  // [0] wait error, [1] merge role
  const int ntile = min(a.tpc, (n_valid + QA_TK - 1) / QA_TK - tile0);
  const int nw = ntile > warp ? (ntile - warp + QA_WARPS - 1) / QA_WARPS : 0;  // warp's tiles

  uint64_t* mbar_m = reinterpret_cast<uint64_t*>(sm + QA_OFF_MBAR);
  if (threadIdx.x == 0) {
    s_flag[0] = 0;
    mbar_init(mbar_m, 1);
  }
  if (lane == 0) {
    for (int s = 0; s < QA_STAGES; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  uint64_t pol = 0;
  // warp w takes the CTA's tiles w, w + 8, w + 16, ...; its j-th goes to stage j % QA_STAGES
  auto issue = [&](int j, int s, int dep) {
    const int row = head_row0 + QA_TK * (tile0 + warp + QA_WARPS * j) + dep;
    mbar_arrive_expect_tx(&bars[s], 2 * QA_TILE + (SC_TMA ? 4 * QA_SC : 0));
    uint8_t* kv = kvw + s * 2 * QA_TILE;
    tma_load_2d_hint(kv, &mp.k, &bars[s], 0, row, pol);
    tma_load_2d_hint(kv + QA_TILE, &mp.v, &bars[s], 0, row, pol);
    if (SC_TMA) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        tma_load_2d(scw + s * 4 * QA_SCS + q * QA_SCS, &mp.s[q], &bars[s], 0, row >> 2);
    }
  };
  // With a device-side length the kernel may start before its predecessor (the prologue that
  // appends the newest key) finishes: the first stages of every tile but the one holding that
  // row stream before the wait; the rest, and q, follow it.
  const int last_tile = (n_valid - 1) / QA_TK;
  auto early = [&](int j) { return a.early && tile0 + warp + QA_WARPS * j != last_tile; };
  if (lane == 0) {
    pol = l2_evict_first_policy();
    for (int j = 0; j < QA_STAGES && j < nw; ++j)
      if (early(j)) issue(j, j, 0);
  }
  pdl_wait();
  pdl_trigger();
  if (lane == 0)
    for (int j = 0; j < QA_STAGES && j < nw; ++j)
      if (!early(j)) issue(j, j, 0);

  // ---- Q^T fragments (B operand of S^T = K Q^T): column n = head r (+ 8 nt) ----
  // k-block kb (group g = kb / 4, word wi = kb % 4) covers dims 64g + 16c4 + 4wi + {0..3}
  uint32_t qb[NT][8][2];
  float qs[NT][2][2];  // sum over group g of the fp16-rounded q of heads 2c4 + hh (+ 8 nt)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = r + 8 * nt;
    const bool hv = h < G;
    const __nv_bfloat16* qrow = a.q + ((size_t)b * a.Hq + hk * G + (hv ? h : 0)) * QA_D;
    float qsum[2];
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
        qb[nt][4 * g + wi][0] = pack_h2(v[0], v[1]);
        qb[nt][4 * g + wi][1] = pack_h2(v[2], v[3]);
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      qsum[g] = s;
    }
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        qs[nt][g][hh] = __shfl_sync(0xffffffffu, qsum[g], (2 * c4 + hh) * 4);
  }

  const int kr0 = kperm(r), kr1 = kr0 + 8;                  // keys of S^T rows r, r + 8
  const int vk0 = kperm(2 * c4), vk1 = kperm(2 * c4 + 1);    // keys of P'^T rows 2c4, 2c4+1

  float m[NT][2], l[NT][2], ob[NT][2][2], acc[NT][8][4], c1[NT][2][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      m[nt][hh] = -INFINITY;
      l[nt][hh] = 0.f;
      ob[nt][0][hh] = ob[nt][1][hh] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[nt][i][0] = acc[nt][i][1] = acc[nt][i][2] = acc[nt][i][3] = 0.f;
#pragma unroll
    for (int g = 0; g < 2; ++g) c1[nt][g][0] = c1[nt][g][1] = c1[nt][g][2] = c1[nt][g][3] = 0.f;
  }

  int j = 0;
  for (; j < nw; ++j) {
    const int s = j % QA_STAGES;
    const int t0 = QA_TK * (tile0 + warp + QA_WARPS * j);
    // the warp leaves together: the loop body issues warp-collective MMAs
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (j / QA_STAGES) & 1, s_flag, 1))) break;
    const uint8_t* Kt = kvw + s * 2 * QA_TILE;
    const uint8_t* Vt = Kt + QA_TILE;
    uint8_t* St = scw + s * 4 * QA_SCS;
    if (!SC_TMA) {  // scale arrays not 16-byte addressable per tile: plain loads
      const size_t row = (size_t)head_row0 + min(t0 + lane, n_valid - 1);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<uint32_t*>(St + q * QA_SCS)[lane] = __ldg(a.sc[q] + row);
      __syncwarp();
    }

    // ---- every shared-memory read of this stage, then its refill ----
    // half hf holds keys 16 hf .. 16 hf + 15 of the tile
    uint4 kw[2][2][2];  // [half][key kr0 / kr1][head-dim group]
    uint2 vw[2][4][2];  // [half][key vk0, vk1, vk0 + 8, vk1 + 8][group]: bytes 64g + 8r .. + 7
    uint32_t scw4[2][2][4];  // [half][key kr0 / kr1][ks, kb, vs, vb] words {g0, g1}
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int g = 0; g < 2; ++g)
          kw[hf][i][g] =
              *reinterpret_cast<const uint4*>(Kt + sw128(16 * hf + (i ? kr1 : kr0), 4 * g + c4));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int key = 16 * hf + (q & 1 ? vk1 : vk0) + (q & 2 ? 8 : 0);
#pragma unroll
        for (int g = 0; g < 2; ++g)
          vw[hf][q][g] =
              *reinterpret_cast<const uint2*>(Vt + sw128(key, 4 * g + (r >> 1)) + 8 * (r & 1));
      }
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          scw4[hf][i][q] =
              *reinterpret_cast<const uint32_t*>(St + q * QA_SCS + 4 * (16 * hf + (i ? kr1 : kr0)));
    }
    {
      // The warp-wide XOR consumes every loaded register of every lane, and the refill's row
      // coordinate depends on it (times a runtime zero), so the TMA cannot overwrite this
      // stage before all of its reads have landed.
      uint32_t dep = 0;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int g = 0; g < 2; ++g)
            dep ^= kw[hf][i][g].x ^ kw[hf][i][g].y ^ kw[hf][i][g].z ^ kw[hf][i][g].w;
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int g = 0; g < 2; ++g) dep ^= vw[hf][q][g].x ^ vw[hf][q][g].y;
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) dep ^= scw4[hf][i][q];
      }
      const uint32_t gate = __reduce_xor_sync(0xffffffffu, dep);
      if (lane == 0 && j + QA_STAGES < nw) {
        fence_proxy_async_smem();
        issue(j + QA_STAGES, s, static_cast<int>(gate) * a.zero);
      }
    }
    __syncwarp();  // rejoin the warp (lane 0's refill, the per-lane stage wait) before the MMAs

    // ---- S^T = K Q^T per half (two accumulators: head-dim groups 0 and 1) ----
    float sa[2][NT][2][4];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int g = 0; g < 2; ++g)
          sa[hf][nt][g][0] = sa[hf][nt][g][1] = sa[hf][nt][g][2] = sa[hf][nt][g][3] = 0.f;
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
      const int g = kb >> 2, wi = kb & 3;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint32_t w0 = u4get(kw[hf][0][g], wi), w1 = u4get(kw[hf][1][g], wi);
        const uint32_t a0 = code_h2(w0, 0x4140u), a1 = code_h2(w1, 0x4140u);
        const uint32_t a2 = code_h2(w0, 0x4342u), a3 = code_h2(w1, 0x4342u);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma_f16(sa[hf][nt][g], a0, a1, a2, a3, qb[nt][kb][0], qb[nt][kb][1]);
      }
    }

    // ---- scales of keys kr0 / kr1 per half; masked keys get zero V scale and bias ----
    float ksf[2][2][2], kbf[2][2][2], vsf[2][2][2], vbf[2][2][2];  // [half][key][group]
    bool valid[2][2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        valid[hf][i] = t0 + 16 * hf + (i ? kr1 : kr0) < k_end;
        const uint32_t ksw = scw4[hf][i][0], kbw = scw4[hf][i][1];
        const uint32_t vsw = scw4[hf][i][2], vbw = scw4[hf][i][3];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float ks = g ? bfh(ksw) : bfl(ksw);
          ksf[hf][i][g] = ks;
          kbf[hf][i][g] = (g ? bfh(kbw) : bfl(kbw)) - 1024.f * ks;  // removes the code offset
          vsf[hf][i][g] = valid[hf][i] ? (g ? bfh(vsw) : bfl(vsw)) * QA_PSCALE : 0.f;
          vbf[hf][i][g] = valid[hf][i] ? (g ? bfh(vbw) : bfl(vbw)) : 0.f;
        }
      }

    // ---- scores, one online-softmax step for both halves (columns = heads 2c4+hh+8nt) ----
    float p[2][NT][2][2], corr[NT][2];  // p[half][nt][key][head]
    bool rescale = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float sc[2][2][2];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float v = ksf[hf][i][0] * sa[hf][nt][0][2 * i + hh] +
                            ksf[hf][i][1] * sa[hf][nt][1][2 * i + hh] +
                            kbf[hf][i][0] * qs[nt][0][hh] + kbf[hf][i][1] * qs[nt][1][hh];
            sc[hf][i][hh] = valid[hf][i] ? v : -INFINITY;
          }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float mx = fmaxf(fmaxf(sc[0][0][hh], sc[0][1][hh]), fmaxf(sc[1][0][hh], sc[1][1][hh]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[nt][hh], mx);
        const float ref = (mn == -INFINITY) ? 0.f : mn;
        const float cr = ex2(m[nt][hh] - ref);
        rescale |= (cr != 1.f);
        corr[nt][hh] = cr;
        m[nt][hh] = mn;
        float ls = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float pv = ex2(sc[hf][i][hh] - ref);
            p[hf][nt][i][hh] = pv;
            ls += pv;
            o0 += pv * vbf[hf][i][0];
            o1 += pv * vbf[hf][i][1];
          }
        l[nt][hh] = l[nt][hh] * cr + ls;
        ob[nt][0][hh] = ob[nt][0][hh] * cr + o0;
        ob[nt][1][hh] = ob[nt][1][hh] * cr + o1;
      }
    }
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[nt][i][0] *= corr[nt][0];
          acc[nt][i][1] *= corr[nt][1];
          acc[nt][i][2] *= corr[nt][0];
          acc[nt][i][3] *= corr[nt][1];
        }
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          c1[nt][g][0] *= corr[nt][0];
          c1[nt][g][1] *= corr[nt][1];
          c1[nt][g][2] *= corr[nt][0];
          c1[nt][g][3] *= corr[nt][1];
        }
      }
    }

    // ---- P' = p * vs * 256 (fp16), moved into the B layout of O^T = V^T P'^T ----
    uint32_t bp[2][NT][2][2];  // [half][nt][group][b0 / b1]
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          bp[hf][nt][g][0] = movtrans(pack_h2(p[hf][nt][0][0] * vsf[hf][0][g],
                                              p[hf][nt][0][1] * vsf[hf][0][g]));
          bp[hf][nt][g][1] = movtrans(pack_h2(p[hf][nt][1][0] * vsf[hf][1][g],
                                              p[hf][nt][1][1] * vsf[hf][1][g]));
        }

    // ---- O^T += V^T P'^T: M tile mt covers dims 64g + 8r + 2(mt % 4) + {0 (row r), 1 (r+8)} ----
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int g = mt >> 2, jw = (mt >> 1) & 1;
      const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;  // interleave bytes {0,1} or {2,3}
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint32_t tA = prmt32(jw ? vw[hf][0][g].y : vw[hf][0][g].x,
                                   jw ? vw[hf][1][g].y : vw[hf][1][g].x, sel);
        const uint32_t tB = prmt32(jw ? vw[hf][2][g].y : vw[hf][2][g].x,
                                   jw ? vw[hf][3][g].y : vw[hf][3][g].x, sel);
        const uint32_t a0 = code_h2(tA, 0x4140u), a1 = code_h2(tA, 0x4342u);
        const uint32_t a2 = code_h2(tB, 0x4140u), a3 = code_h2(tB, 0x4342u);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma_f16(acc[nt][mt], a0, a1, a2, a3, bp[hf][nt][g][0], bp[hf][nt][g][1]);
      }
    }
    constexpr uint32_t ONE2 = 0x3C003C00u;  // fp16x2 {1, 1}
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int g = 0; g < 2; ++g)
          mma_f16(c1[nt][g], ONE2, ONE2, ONE2, ONE2, bp[hf][nt][g][0], bp[hf][nt][g][1]);
  }
  if (j < nw) {
    // a wait gave up: drain this warp's other loads in flight (bounded) before leaving
    for (int jj = j + 1; jj < nw && jj < j + QA_STAGES; ++jj)
      mbar_wait(&bars[jj % QA_STAGES], (jj / QA_STAGES) & 1, s_flag, 1, 200000000LL);
  }

  // ---- row sums and bias terms over this warp's keys (lanes with the same c4) ----
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l[nt][hh] += __shfl_xor_sync(0xffffffffu, l[nt][hh], o);
        ob[nt][0][hh] += __shfl_xor_sync(0xffffffffu, ob[nt][0][hh], o);
        ob[nt][1][hh] += __shfl_xor_sync(0xffffffffu, ob[nt][1][hh], o);
      }
    }
  __syncthreads();  // every warp is done with its ring: reuse it for the warp outputs
  float* slab = reinterpret_cast<float*>(sm + QA_OFF_SLAB);  // [warp][16][128]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int head = 2 * c4 + hh + 8 * nt;
      if (head < G) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int g = mt >> 2;
          const float base = ob[nt][g][hh] - (1024.f / QA_PSCALE) * c1[nt][g][hh];
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int d = 64 * g + 8 * r + 2 * (mt & 3) + h2;
            slab[(warp * 16 + head) * QA_SLAB + d] = acc[nt][mt][2 * h2 + hh] * (1.f / QA_PSCALE) + base;
          }
        }
        if (r == 0) {
          s_m[warp * 16 + head] = m[nt][hh];
          s_l[warp * 16 + head] = l[nt][hh];
        }
      }
    }
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < QA_WARPS; ++w) M = fmaxf(M, s_m[w * 16 + h]);
    float L = 0.f;
    for (int w = 0; w < QA_WARPS; ++w) {
      const float mw = s_m[w * 16 + h];
      const float wt = (mw == -INFINITY) ? 0.f : ex2(mw - M);
      s_wt[w * 16 + h] = wt;
      L += wt * s_l[w * 16 + h];
    }
    s_M[h] = M;
    s_L[h] = L;
  }
  __syncthreads();
  const int ns = a.nsplit;
  if (ns == 1) {  // the CTA owns the whole (batch, kv head): write the output directly
    const bool bad = s_flag[0] != 0;
    for (int i = threadIdx.x; i < G * (QA_D / 2); i += QA_THREADS) {
      const int h = i / (QA_D / 2), d = 2 * (i % (QA_D / 2));
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < QA_WARPS; ++w) {
        v0 += s_wt[w * 16 + h] * slab[(w * 16 + h) * QA_SLAB + d];
        v1 += s_wt[w * 16 + h] * slab[(w * 16 + h) * QA_SLAB + d + 1];
      }
      const float inv = 1.f / s_L[h];
      if (bad) v0 = v1 = __int_as_float(0x7fc00000);
      const size_t head = (size_t)b * a.Hq + hk * G + h;
      *reinterpret_cast<__nv_bfloat162*>(a.out + head * QA_D + d) =
          __floats2bfloat162_rn(q8_gated(v0 * inv, a, head), q8_gated(v1 * inv, a, head));
    }
    return;
  }
  // ---- this CTA's partial: (max, sum) and the weighted accumulator per head ----
  const size_t mls = (size_t)q8_ml_stride(ns, G);
  const size_t pbase = ((size_t)bh * ns + split) * G;
  for (int i = threadIdx.x; i < G * QA_D; i += QA_THREADS) {
    const int h = i / QA_D, d = i % QA_D;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < QA_WARPS; ++w) v += s_wt[w * 16 + h] * slab[(w * 16 + h) * QA_SLAB + d];
    a.part_acc[(pbase + h) * QA_D + d] = v;
  }
  if (threadIdx.x < G)
    a.part_ml[bh * mls + split * G + threadIdx.x] = make_float2(s_M[threadIdx.x], s_L[threadIdx.x]);

  // ---- the last CTA of this (batch, kv head) merges every split ----
  __syncthreads();  // this split's partials are stored before thread 0 releases them
  if (threadIdx.x == 0) {
    const int add = 1 + (s_flag[0] ? (1 << 20) : 0);
    const int total = atom_add_acq_rel_gpu(&a.counters[bh * 32], add) + add;
    s_flag[1] = ((total & 0xFFFFF) == ns) ? ((total >> 20) ? 2 : 1) : 0;
  }
  __syncthreads();  // the merger: every split's partials, acquired by thread 0, are visible
  if (s_flag[1] == 0) return;
  const int nsg = ns * G;
  const float2* gml = a.part_ml + bh * mls;
  const float* gacc = a.part_acc + (size_t)bh * nsg * QA_D;
  const bool whole = nsg <= QA_MERGE_SMEM;
  float* t_acc = reinterpret_cast<float*>(sm);  // [split][G][D] (whole copy only)
  const size_t acc_bytes = whole ? (size_t)nsg * QA_D * 4 : 0;
  float2* t_ml = reinterpret_cast<float2*>(sm + acc_bytes);  // [split][G]
  const uint32_t ml_bytes = (uint32_t)(mls * sizeof(float2));
  float* t_w = reinterpret_cast<float*>(sm + acc_bytes + ml_bytes);  // [split][G]
  bool ok = true;
  if (whole) {
    // every split's partial of this head into shared memory with one bulk copy
    if (threadIdx.x == 0) {
      fence_proxy_async_global();  // the other CTAs' partials (acquired above) to the copy
      mbar_arrive_expect_tx(mbar_m, (uint32_t)acc_bytes + ml_bytes);
      bulk_g2s(t_acc, gacc, (uint32_t)acc_bytes, mbar_m);
      bulk_g2s(t_ml, gml, ml_bytes, mbar_m);
    }
    ok = mbar_wait(mbar_m, 0, s_flag, 2);
  } else {
    for (int i = threadIdx.x; i < nsg; i += QA_THREADS) t_ml[i] = __ldcg(gml + i);
  }
  ok = __syncthreads_and(ok);  // one verdict for the whole CTA
  // per head (one warp each): max over splits, then the normalised split weights
  for (int h = warp; h < G; h += QA_WARPS) {
    float M = -INFINITY;
    for (int s = lane; s < ns; s += 32) M = fmaxf(M, t_ml[s * G + h].x);
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < ns; s += 32) {
      const float2 v = t_ml[s * G + h];
      const float w = (v.x == -INFINITY) ? 0.f : ex2(v.x - M);
      t_w[s * G + h] = w;
      L += v.y * w;
    }
    L = warp_sum(L);
    const float inv = 1.f / L;
    for (int s = lane; s < ns; s += 32) t_w[s * G + h] *= inv;
  }
  __syncthreads();
  const bool bad = s_flag[1] == 2 || !ok;
  // one item = 4 dims of one head
  for (int it = threadIdx.x; it < G * (QA_D / 4); it += QA_THREADS) {
    const int h = it / (QA_D / 4), d4 = it % (QA_D / 4);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (whole) {
      const float4* src = reinterpret_cast<const float4*>(t_acc) + h * (QA_D / 4) + d4;
#pragma unroll 4
      for (int s = 0; s < ns; ++s) {
        const float w = t_w[s * G + h];
        const float4 v = src[(size_t)s * G * (QA_D / 4)];
        o.x += w * v.x;
        o.y += w * v.y;
        o.z += w * v.z;
        o.w += w * v.w;
      }
    } else {
      const float4* src = reinterpret_cast<const float4*>(gacc) + h * (QA_D / 4) + d4;
      constexpr int MB = 8;  // loads in flight per thread
      for (int s0 = 0; s0 < ns; s0 += MB) {
        float4 v[MB];
#pragma unroll
        for (int u = 0; u < MB; ++u)
          if (s0 + u < ns) v[u] = __ldcg(src + (size_t)(s0 + u) * G * (QA_D / 4));
#pragma unroll
        for (int u = 0; u < MB; ++u)
          if (s0 + u < ns) {
            const float w = t_w[(s0 + u) * G + h];
            o.x += w * v[u].x;
            o.y += w * v[u].y;
            o.z += w * v[u].z;
            o.w += w * v[u].w;
          }
      }
    }
    if (bad) o.x = o.y = o.z = o.w = __int_as_float(0x7fc00000);
    const size_t head = (size_t)b * a.Hq + hk * G + h;
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(a.out + head * QA_D + 4 * d4);
    dst[0] = __floats2bfloat162_rn(q8_gated(o.x, a, head), q8_gated(o.y, a, head));
    dst[1] = __floats2bfloat162_rn(q8_gated(o.z, a, head), q8_gated(o.w, a, head));
  }
  if (threadIdx.x == 0) a.counters[bh * 32] = 0;  // leave the counter at zero for the next call
}

// CTAs per (batch, kv head): one CTA per SM is resident (the rings take ~207 KB), so fill the
// SMs once, each CTA a contiguous range of whole 32-key tiles, with at least one tile per
// warp. B * Hkv > 74 leaves one CTA per (batch, kv head) (no split merge).
static int q8_sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return 148;  // no device (host-side size queries): a B200
  }
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

static void q8_split(int B, int Hkv, int n, int* tpc, int* nsplit) {
  const int BH = B * Hkv;
  const int SMS = q8_sm_count();
  const int nt = (n + QA_TK - 1) / QA_TK;
  int ns = SMS / BH;
  ns = min(ns, (nt + QA_WARPS - 1) / QA_WARPS);
  ns = max(1, min(ns, QA_MAX_SPLITS));
  const int t = (nt + ns - 1) / ns;
  *tpc = t;
  *nsplit = (nt + t - 1) / t;
}

// Workspace: a fixed control region (one 128-byte counter slot per (batch, kv head); only
// splits > 1 use it, which implies B * Hkv <= 74) that must start zeroed and is left zeroed by
// every completed call, then the split partials. The control region's place and size do not
// depend on the call, so calls of any shapes can share one workspace.
constexpr size_t QA_CTRL_BYTES = 16384;
constexpr int QA_CTRL_SLOTS = (int)(QA_CTRL_BYTES / 128);

struct Q8Ws {
  size_t ml, acc, total;
};

static Q8Ws q8_layout(int B, int Hq, int Hkv, int n) {
  int tpc, ns;
  q8_split(B, Hkv, n < 1 ? 1 : n, &tpc, &ns);
  const size_t G = (size_t)Hq / (Hkv > 0 ? Hkv : 1);
  const size_t parts = (size_t)B * Hkv * ns * G;
  const size_t mls = (size_t)q8_ml_stride(ns, (int)G);
  Q8Ws w;
  w.ml = QA_CTRL_BYTES;
  w.acc = w.ml + (ns > 1 ? align_up(sizeof(float2) * (size_t)B * Hkv * mls, 256) : 0);
  w.total = w.acc + (ns > 1 ? align_up(sizeof(float) * parts * QA_D, 256) : 0);
  return w;
}

static size_t q8_ws(int B, int Hq, int Hkv, int n, size_t* counters_bytes) {
  const Q8Ws w = q8_layout(B, Hq, Hkv, n);
  if (counters_bytes) *counters_bytes = QA_CTRL_BYTES;
  return w.total;
}

// Tensor maps depend only on the cache buffers and their row count; a decode loop reuses
// the same buffers call after call, so keep the last few encodings.
struct Q8MapKey {
  const void* p[6];
  long long rows;
  bool sc_tma;
  int dev;
};

static int q8_maps(const Q8MapKey& key, Q8Maps* out) {
  constexpr int CACHE = 64;
  static std::mutex mu;
  static Q8MapKey keys[CACHE];
  static Q8Maps maps[CACHE];
  static int used = 0, next = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i) {
    const Q8MapKey& k = keys[i];
    bool same = k.rows == key.rows && k.sc_tma == key.sc_tma && k.dev == key.dev;
    for (int t = 0; t < 6 && same; ++t) same = k.p[t] == key.p[t];
    if (same) {
      *out = maps[i];
      return LG_OK;
    }
  }
  Q8Maps m;
  int rc;
  if ((rc = make_map_2d(&m.k, key.p[0], false, 32, key.rows, 128, 32, QA_TK, 128))) return rc;
  if ((rc = make_map_2d(&m.v, key.p[1], false, 32, key.rows, 128, 32, QA_TK, 128))) return rc;
  for (int q = 0; q < 4; ++q) {
    if (key.sc_tma) {
      if ((rc = make_map_2d(&m.s[q], key.p[2 + q], true, 8, key.rows / 4, 16, 8, QA_TK / 4, 0)))
        return rc;
    } else {
      m.s[q] = m.k;  // never read
    }
  }
  const int slot = used < CACHE ? used++ : (next++ % CACHE);
  keys[slot] = key;
  maps[slot] = m;
  *out = m;
  return LG_OK;
}

struct Q8Call {
  const __nv_bfloat16* q;
  const uint32_t *kq, *vq;
  const void* sc[4];  // ks, kb, vs, vb
  int B, Hq, Hkv, cap, n;
  __nv_bfloat16* out;
  const int* n_dev = nullptr;  // device-side length (*n_dev + n_add), planned for n
  int n_add = 0;
  const __nv_bfloat16* gate = nullptr;
};

template <int NT, bool SCT>
static int q8_launch_one(dim3 grid, const Q8Maps& mp, const Q8Args& a, cudaStream_t st) {
  static unsigned long long attr_done = 0;  // bit per device
  int dev = 0;
  LG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !((attr_done >> dev) & 1ull)) {
    LG_CUDA_TRY(cudaFuncSetAttribute(q8_decode_kernel<NT, SCT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, QA_SMEM));
    attr_done |= 1ull << dev;
  }
  LG_CUDA_TRY(launch_k(q8_decode_kernel<NT, SCT>, grid, dim3(QA_THREADS), QA_SMEM, st, mp, a));
  return LG_OK;
}

int launch_q8_decode(const Q8Call& c, float scale, void* ws, cudaStream_t st) {
  Q8Args a;
  a.q = c.q;
  for (int i = 0; i < 4; ++i) a.sc[i] = static_cast<const uint32_t*>(c.sc[i]);
  a.B = c.B;
  a.Hq = c.Hq;
  a.Hkv = c.Hkv;
  a.G = c.Hq / c.Hkv;
  a.cap = c.cap;
  a.n = c.n;
  a.out = c.out;
  a.n_dev = c.n_dev;
  a.n_add = c.n_add;
  a.gate = c.gate;
  a.early = c.n_dev != nullptr;
  q8_split(a.B, a.Hkv, a.n, &a.tpc, &a.nsplit);
  if (a.nsplit > 1 && a.B * a.Hkv > QA_CTRL_SLOTS)
    return fail(LG_ERR_UNSUPPORTED, "q8 decode: %d splits for %d (batch, kv head) pairs",
                a.nsplit, a.B * a.Hkv);
  a.zero = 0;
  a.qscale = scale * 1.4426950408889634f;
  const Q8Ws w = q8_layout(c.B, c.Hq, c.Hkv, c.n);
  char* base = static_cast<char*>(ws);
  a.counters = reinterpret_cast<int*>(base);
  a.part_ml = reinterpret_cast<float2*>(base + w.ml);
  a.part_acc = reinterpret_cast<float*>(base + w.acc);

  Q8MapKey key;
  key.p[0] = c.kq;
  key.p[1] = c.vq;
  bool sct = (c.cap % 4) == 0;
  for (int i = 0; i < 4; ++i) {
    key.p[2 + i] = c.sc[i];
    sct = sct && aligned(c.sc[i], 16);
  }
  key.rows = (long long)c.B * c.Hkv * c.cap;
  key.sc_tma = sct;
  LG_CUDA_TRY(cudaGetDevice(&key.dev));
  Q8Maps mp;
  int rc = q8_maps(key, &mp);
  if (rc) return rc;

  dim3 grid(a.nsplit, a.Hkv, a.B);
  prof_begin("q8_decode", st);
  if (a.G <= 8)
    rc = sct ? q8_launch_one<1, true>(grid, mp, a, st) : q8_launch_one<1, false>(grid, mp, a, st);
  else
    rc = sct ? q8_launch_one<2, true>(grid, mp, a, st) : q8_launch_one<2, false>(grid, mp, a, st);
  if (rc) return rc;
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
  LG_CHECK_ARG((long long)B * Hkv * cap < (1LL << 31),
               "q8 decode: B * Hkv * cap = %lld rows exceeds 2^31", (long long)B * Hkv * cap);
  LG_CHECK_ARG(q && k_q && k_s && k_b && v_q && v_s && v_b && out, "q8 decode: NULL pointer");
  LG_CHECK_ARG(aligned(k_q, 16) && aligned(v_q, 16) && aligned(k_s, 4) && aligned(k_b, 4) &&
                   aligned(v_s, 4) && aligned(v_b, 4) && aligned(q, 4) && aligned(out, 8),
               "q8 decode: packed K/V must be 16-byte aligned, scales/biases and q 4-byte, "
               "out 8-byte aligned");
  return LG_OK;
}

static Q8Call make_call(const void* q, int B, int Hq, int Hkv, const uint32_t* k_q,
                        const void* k_s, const void* k_b, const uint32_t* v_q, const void* v_s,
                        const void* v_b, int cap, int n, void* out) {
  Q8Call c;
  c.q = static_cast<const __nv_bfloat16*>(q);
  c.kq = k_q;
  c.vq = v_q;
  c.sc[0] = k_s;
  c.sc[1] = k_b;
  c.sc[2] = v_s;
  c.sc[3] = v_b;
  c.B = B;
  c.Hq = Hq;
  c.Hkv = Hkv;
  c.cap = cap;
  c.n = n;
  c.out = static_cast<__nv_bfloat16*>(out);
  return c;
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
  const size_t need = q8_ws(B, Hq, Hkv, n, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "q8 decode: workspace %zu bytes at %p, need %zu (256-aligned)",
                workspace_bytes, workspace, need);
  return launch_q8_decode(make_call(q, B, Hq, Hkv, k_q, k_s, k_b, v_q, v_s, v_b, cap, n, out),
                          scale, workspace, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
// Fixed-scratch variant: the same kernel with its split partials and completion counters in
// a file-scope device array instead of a caller workspace, for callers that cannot allocate
// device memory when they call. The array's device address is looked up once per device
// with cudaGetSymbolAddress (in host code the symbol name is only a stand-in).
// ---------------------------------------------------------------------------------------
namespace lg {

constexpr size_t Q8_FIXED_SCRATCH_BYTES = (size_t)1 << 20;  // 1 MiB per device
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
  return launch_q8_decode(make_call(q, B, Hq, Hkv, k_q, k_s, k_b, v_q, v_s, v_b, cap, n, out),
                          scale, base, st);
}

extern "C" int lg_q8_decode_attention_dev(const void* q, int B, int Hq, int Hkv, int D,
                                          const uint32_t* k_q, const void* k_s, const void* k_b,
                                          const uint32_t* v_q, const void* v_s, const void* v_b,
                                          int cap, int n_plan, const int32_t* n_dev, int n_add,
                                          float scale, const void* gate, void* out,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_q8_args(q, B, Hq, Hkv, D, k_q, k_s, k_b, v_q, v_s, v_b, cap, n_plan, out);
  if (rc) return rc;
  LG_CHECK_ARG(n_dev != nullptr, "q8 decode: n_dev is NULL (use lg_q8_decode_attention)");
  LG_CHECK_ARG(!gate || aligned(gate, 2), "q8 decode: gate must be 2-byte aligned");
  const size_t need = lg_q8_decode_workspace_bytes(B, Hq, Hkv, n_plan);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "q8 decode: workspace needs %zu bytes (256-aligned)", need);
  Q8Call c = make_call(q, B, Hq, Hkv, k_q, k_s, k_b, v_q, v_s, v_b, cap, n_plan, out);
  c.n_dev = n_dev;
  c.n_add = n_add;
  c.gate = static_cast<const __nv_bfloat16*>(gate);
  return launch_q8_decode(c, scale, workspace, static_cast<cudaStream_t>(stream));
}
