// bs1 decode chain: a token's dense linears, router and MoE experts as few kernels, each of
// which streams its weights into shared memory with bulk copies (issued before its PDL wait
// wherever the weights do not depend on the previous kernel) and fuses the elementwise work
// around it.
//
//  dgemv_kernel          y = W x (4-bit g64, laguna.py:84-92) for one token, with the input
//                        RMSNorm fused in front (the decoder layer's norms, laguna.py:158-161,
//                        :189), an optional residual add, or a gate/up pair with the SwiGLU of
//                        laguna.py:122 (the dense MLP of layer 0).
//  router_decode_kernel  post-attention RMSNorm + 8-bit router logits + sigmoid / bias /
//                        top-k / renormalisation (laguna.py:137-145) for one token in one CTA
//                        that holds the whole router weight in shared memory.
//  moe_dec_gateup_kernel gate/up products of the k picked experts and the shared expert with
//                        the SwiGLU epilogue (SwitchGLU, laguna.py:149; MLP, :114-122).
//  moe_dec_down_kernel   down products of all k + 1 groups for a 16-row slice of the hidden
//                        dimension, the weighted combine (laguna.py:149-150) and the residual
//                        add, in a fixed order (no atomics).
//
// Arithmetic per 64-group is the tensor-core group product of gemv_core.cuh with the affine
// dequantisation folded in per group (scale * sum(code * x) + bias * sum(x)).
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "decode_core.cuh"
#include "gemv_core.cuh"
#include "prep_core.cuh"
#include "tc_ptx.cuh"

namespace lg {

constexpr int DG_MAX_STAGES = 8;

template <int V>
__device__ __forceinline__ void load_sb(const __nv_bfloat16* p, float (&o)[V]) {
  if constexpr (V == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    o[0] = bf_lo(v.x); o[1] = bf_hi(v.x); o[2] = bf_lo(v.y); o[3] = bf_hi(v.y);
    o[4] = bf_lo(v.z); o[5] = bf_hi(v.z); o[6] = bf_lo(v.w); o[7] = bf_hi(v.w);
  } else if constexpr (V == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    o[0] = bf_lo(v.x); o[1] = bf_hi(v.x); o[2] = bf_lo(v.y); o[3] = bf_hi(v.y);
  } else if constexpr (V == 2) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
    o[0] = bf_lo(v); o[1] = bf_hi(v);
  } else {
    o[0] = bf2f(*p);
  }
}

// A warp's share of one staged 16-row tile against one token: groups [g0, g0 + n) (n a
// multiple of V). s0p/s8p/b0p/b8p: scale and bias rows of the thread's rows r and r + 8
// (shared memory, or global for a partial tile). xs: the token's activations (uint4 = 8 bf16),
// gsum: its per-group sums. Lanes with lane % 4 == 0 end with y[r] in y0 and y[r + 8] in y8.
template <int V>
__device__ __forceinline__ void warp_tile_dot(float& y0, float& y8, const uint8_t* tile,
                                              uint32_t pitch, const __nv_bfloat16* s0p,
                                              const __nv_bfloat16* s8p,
                                              const __nv_bfloat16* b0p,
                                              const __nv_bfloat16* b8p, int g0, int n,
                                              const uint4* xs, const float* gsum, int r,
                                              int c4) {
  for (int i = 0; i < n; i += V) {
    float s0[V], s8[V], b0[V], b8[V];
    load_sb<V>(s0p + g0 + i, s0);
    load_sb<V>(s8p + g0 + i, s8);
    load_sb<V>(b0p + g0 + i, b0);
    load_sb<V>(b8p + g0 + i, b8);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int gg = g0 + i + j;
      uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
      if (r == 0) {
        xa0 = xs[gg * 8 + 2 * c4];
        xa1 = xs[gg * 8 + 2 * c4 + 1];
      }
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      tile_group(d, tile, pitch, gg, r, c4, xa0, xa1);
      const float xg = gsum[gg];
      y0 += s0[j] * d[0] + b0[j] * xg;
      y8 += s8[j] * d[2] + b8[j] * xg;
    }
  }
}

// Scale/bias row pointers of the thread's rows for tile rows [row0, row0 + rows) of a matrix
// whose scales are s/b ([*, gpr] bf16): the staged copy when the tile is full, else global.
struct SbRows {
  const __nv_bfloat16 *s0, *s8, *b0, *b8;
};
__device__ __forceinline__ SbRows sb_rows(const uint8_t* tile, int K, int rows, int row0,
                                          int nrows_total, const __nv_bfloat16* s,
                                          const __nv_bfloat16* b, int r) {
  const int gpr = K / 64;
  SbRows o;
  if (rows == 16) {
    const __nv_bfloat16* ss = reinterpret_cast<const __nv_bfloat16*>(tile + tile_sc_off(K));
    o.s0 = ss + r * gpr;
    o.s8 = ss + (r + 8) * gpr;
    o.b0 = o.s0 + 16 * gpr;
    o.b8 = o.s8 + 16 * gpr;
  } else {
    const int ra = min(row0 + r, nrows_total - 1), rb = min(row0 + r + 8, nrows_total - 1);
    o.s0 = s + (size_t)ra * gpr;
    o.s8 = s + (size_t)rb * gpr;
    o.b0 = b + (size_t)ra * gpr;
    o.b8 = b + (size_t)rb * gpr;
  }
  return o;
}

// Per-group sums of the activations in xs (K/64 groups), the same order as the GEMV kernels'
// in-register sums. Whole block; contains no barrier.
__device__ __forceinline__ void group_sums(const uint4* xs, int gpr, float* gsum) {
  const int c4 = threadIdx.x & 3;
  for (int g0 = 0; g0 < gpr; g0 += blockDim.x / 4) {
    const int g = g0 + threadIdx.x / 4;
    float v = 0.f;
    if (g < gpr) v = xsum16(xs[g * 8 + 2 * c4], xs[g * 8 + 2 * c4 + 1]);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    if (g < gpr && c4 == 0) gsum[g] = v;
  }
}

// ---- dense decode GEMV ------------------------------------------------------------------------

struct DgArgs {
  const __nv_bfloat16* x;       // [K] (the residual stream when norm_w is set)
  const __nv_bfloat16* norm_w;  // [K] RMSNorm weight, or null
  float eps;
  const uint32_t* q[2];         // [N, K/8] words: [0] the linear (or gate), [1] up (GLU)
  const __nv_bfloat16* s[2];    // [N, K/64]
  const __nv_bfloat16* b[2];
  const __nv_bfloat16* res;     // [N] or null (plain mode)
  __nv_bfloat16* out;           // [N]
  int K, N, tiles, stages;
  // attention prologue fused behind the q/k/v/g projection (one tile per CTA, one token; its
  // arguments travel as a second kernel parameter, so the plain variants keep a small one)
  int prep;
  unsigned int* head_cnt;  // [Hq + 2 Hkv] finished tiles per head (zero between calls)
};

// shared memory: red8 [8] | red [2][NM][NW][16] | xs [K] bf16 | gsum [K/64] | ring of stages
__host__ __device__ __forceinline__ uint32_t dg_ring_off(int K, int NW) {
  const uint32_t xs = (32u + 2u * 2u * NW * 16u * 4u + 15u) & ~15u;
  return (xs + 2u * K + 4u * (K / 64) + 127u) & ~127u;
}

// grid: CTAs take tiles blockIdx.x, blockIdx.x + gridDim.x, ...; `stages` tiles in flight.
// NW warps split each tile's K groups. PREP: the attention prologue behind a q/k/v/g projection.
template <bool GLU, int NW, int V, bool PREP>
__device__ __forceinline__ void dgemv_body(const DgArgs& a, const PrepArgs& p) {
  constexpr int NM = GLU ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K, gpr = K / 64, S = a.stages;
  const uint32_t pitch = tile_pitch(K), tb = tile_bytes(K);
  float* red8 = reinterpret_cast<float*>(smem);
  float* red = reinterpret_cast<float*>(smem + 32);
  uint4* xs = reinterpret_cast<uint4*>(smem + ((32u + 2u * 2u * NW * 16u * 4u + 15u) & ~15u));
  float* gsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + 2 * K);
  uint8_t* ring = smem + dg_ring_off(K, NW);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = lane >> 2, c4 = lane & 3;
  const int mine = (a.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t slim = dyn_smem_bytes();
  auto issue = [&](int i) {  // this CTA's i-th tile into stage i % S (one copy group)
    if (i < mine) {
      const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * 16;
      const int rows = min(16, a.N - row0);
      uint8_t* st = ring + (size_t)(i % S) * NM * tb;
#pragma unroll
      for (int m = 0; m < NM; ++m)
        tile_load(st + m * tb, a.q[m], a.s[m], a.b[m], row0, rows, K, pol, smem, slim);
    }
    cp_async_commit();
  };
  // the weights are static: stream the first tiles while the previous kernel finishes
  for (int i = 0; i < S; ++i) issue(i);
  pdl_wait();
  pdl_trigger();
  const uint4* xg = reinterpret_cast<const uint4*>(a.x);
  if (a.norm_w) {
    const float rs = block_rms_scale(xg, K, a.eps, red8);
    const uint4* wg = reinterpret_cast<const uint4*>(a.norm_w);
    for (int i = tid; i < K / 8; i += NW * 32) xs[i] = rms_apply8(xg[i], wg[i], rs);
  } else {
    for (int i = tid; i < K / 8; i += NW * 32) xs[i] = xg[i];
  }
  __syncthreads();
  group_sums(xs, gpr, gsum);
  const int gpw = (gpr + NW - 1) / NW;
  const int gw0 = warp * gpw, gwn = max(0, min(gpr, gw0 + gpw) - gw0);
  for (int i = 0; i < mine; ++i) {
    const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * 16;
    const int rows = min(16, a.N - row0);
    const uint8_t* st = ring + (size_t)(i % S) * NM * tb;
    cp_async_wait(S - 1);  // this thread's copies of tile i have landed
    __syncthreads();       // ... and everyone's (also publishes gsum on the first pass)
    float* rb = red + (i & 1) * NM * NW * 16;
#pragma unroll
    for (int m = 0; m < NM; ++m) {
      const uint8_t* tile = st + m * tb;
      const SbRows sr = sb_rows(tile, K, rows, row0, a.N, a.s[m], a.b[m], r);
      float y0 = 0.f, y8 = 0.f;
      warp_tile_dot<V>(y0, y8, tile, pitch, sr.s0, sr.s8, sr.b0, sr.b8, gw0, gwn, xs, gsum, r,
                       c4);
      if (c4 == 0) {
        rb[(m * NW + warp) * 16 + r] = y0;
        rb[(m * NW + warp) * 16 + r + 8] = y8;
      }
    }
    __syncthreads();  // every warp is done with this stage: refill it
    issue(i + S);
    if (tid < rows) {
      const int n = row0 + tid;
      float v[NM];
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) t += rb[(m * NW + w) * 16 + tid];
        v[m] = t;
      }
      if constexpr (GLU) {
        a.out[n] = swiglu_mlx(v[0], v[1]);
      } else {
        float y = round_bf16(v[0]);  // quantized_matmul output
        if (a.res) y += bf2f(a.res[n]);
        a.out[n] = __float2bfloat16_rn(y);
      }
    }
  }
  cp_async_wait(0);
  if constexpr (PREP) {
    // The projection row [q | k | v | gates] of one token, one 16-row tile per CTA, whose
    // outputs warp 0 stored (tid < rows): gate rows become gates right here; the last CTA of a
    // head (D / 16 tiles) to finish runs that head's prologue on the row its neighbours wrote.
    if (warp != 0) return;
    const int D = p.D, gate0 = (p.Hq + 2 * p.Hkv) * D;
    const int row0 = (int)blockIdx.x * 16;
    if (row0 >= gate0) {
      if (lane < min(16, a.N - row0))
        p.gate_out[row0 + lane - gate0] = prep_gate(bf2f(a.out[row0 + lane]));
      return;
    }
    const int h = row0 / D;
    __syncwarp();  // the tile's stores come before the release below
    unsigned prev = 0;
    if (lane == 0) prev = atom_add_acq_rel_gpu(&a.head_cnt[h], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(D / 16 - 1)) return;
    __syncwarp();  // ... and the other tiles' stores, acquired by lane 0, before the reads
    if (lane == 0) a.head_cnt[h] = 0u;  // ready for the next call
    prep_head(p, 0, h, false, reinterpret_cast<uint8_t*>(xs));
  }
}

template <bool GLU, int NW, int V>
__global__ void __launch_bounds__(NW * 32) dgemv_kernel(DgArgs a) {
  dgemv_body<GLU, NW, V, false>(a, PrepArgs{});
}

// The q/k/v/g projection with the prologue: its tiles must fit the GPU in one wave (the per-head
// counters need no co-residency, but a second wave would add its whole duration), so the
// kernel keeps to three 8-warp CTAs per SM.
template <int V>
__global__ void __launch_bounds__(256, 3) dgemv_prep_kernel(DgArgs a, PrepArgs p) {
  dgemv_body<false, 8, V, true>(a, p);
}

// ---- router ----------------------------------------------------------------------------------

constexpr int RD_WARPS = 8;  // a warp per expert

struct RdArgs {
  const __nv_bfloat16* h;  // [H] residual stream after attention
  const __nv_bfloat16* norm_w;
  float eps;
  const uint32_t* gq;  // 8-bit g64 router weight [E, H/4] words
  const __nv_bfloat16* gs;
  const __nv_bfloat16* gb;
  const float* ebias;  // [E] or null
  int H, E, k, norm, score_fn;
  __nv_bfloat16* xn_out;  // [H] normalised input of the experts
  int32_t* inds;          // [k]
  __nv_bfloat16* wout;    // [k]
  float* logits;          // [E] or null
  float* lg_ws;           // [E] logits of every CTA (workspace)
  unsigned int* counter;  // CTAs done (workspace, zero between calls)
};

// shared memory: red8 [8] | keys [256] | vals [256] | slot [32] | flag | xs [H] bf16 |
// codes [RD_WARPS][H] | scales, biases [RD_WARPS][H/64] | norm weight [H] | bias [256]
__host__ __device__ __forceinline__ uint32_t rd_xs_off() { return 32u + 2u * 1024u + 128u + 16u; }
__host__ __device__ __forceinline__ uint32_t rd_w_off(int H) {
  return (rd_xs_off() + 2u * H + 127u) & ~127u;
}
// then the norm weight [H] bf16 and the selection bias [256] fp32 (both static: staged before
// the wait)
__host__ __device__ __forceinline__ uint32_t rd_nw_off(int H) {
  return rd_w_off(H) + (uint32_t)RD_WARPS * H + 2u * RD_WARPS * (H / 64) * 2u;
}
__host__ __device__ __forceinline__ size_t rd_smem(int H) {
  return rd_nw_off(H) + 2u * (size_t)H + 4u * 256u;
}

// grid ceil(E / RD_WARPS): each CTA streams its experts' router rows into shared memory
// before the wait (they are static), normalises h and computes its logits (a warp per
// expert); the last CTA to finish gathers all logits and runs the top-k.
__global__ void __launch_bounds__(RD_WARPS * 32) router_decode_kernel(RdArgs a) {
  constexpr int NT = RD_WARPS * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red8 = reinterpret_cast<float*>(smem);
  float* keys = reinterpret_cast<float*>(smem + 32);
  float* vals = keys + 256;
  int* slot = reinterpret_cast<int*>(vals + 256);
  int* flag = slot + 32;
  uint4* xs = reinterpret_cast<uint4*>(smem + rd_xs_off());
  const int H = a.H, E = a.E, gpr = H / 64;
  uint8_t* wq = smem + rd_w_off(H);
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(wq + (size_t)RD_WARPS * H);
  __nv_bfloat16* wb = ws + RD_WARPS * gpr;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int e0 = blockIdx.x * RD_WARPS, ne = min(RD_WARPS, E - e0);
  {
    const uint64_t pol = l2_evict_first_policy();
    const uint32_t slim = dyn_smem_bytes();
    const int cb = ne * H / 16, sb = ne * gpr * 2 / 16;  // 16-byte chunks
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.gq) + (size_t)e0 * H;
    for (int c = tid; c < cb; c += NT)
      cp_async16(wq + c * 16, src + (size_t)c * 16, pol, smem, slim);
    const uint8_t* ss = reinterpret_cast<const uint8_t*>(a.gs + (size_t)e0 * gpr);
    const uint8_t* sbp = reinterpret_cast<const uint8_t*>(a.gb + (size_t)e0 * gpr);
    for (int c = tid; c < 2 * sb; c += NT)
      cp_async16((c < sb ? reinterpret_cast<uint8_t*>(ws) : reinterpret_cast<uint8_t*>(wb) -
                                                                sb * 16) + c * 16,
                 (c < sb ? ss : sbp - sb * 16) + c * 16, pol, smem, slim);
    const uint8_t* nsrc = reinterpret_cast<const uint8_t*>(a.norm_w);
    for (int c = tid; c < H / 8; c += NT)
      cp_async16(smem + rd_nw_off(H) + c * 16, nsrc + (size_t)c * 16, pol, smem, slim);
    cp_async_commit();
  }
  float* ebs = reinterpret_cast<float*>(smem + rd_nw_off(H) + 2 * H);  // [E] selection bias
  for (int e = tid; e < E; e += NT) ebs[e] = a.ebias ? a.ebias[e] : 0.f;
  pdl_wait();
  pdl_trigger();
  const uint4* hg = reinterpret_cast<const uint4*>(a.h);
  const float rs = block_rms_scale(hg, H, a.eps, red8);
  const uint4* nw = reinterpret_cast<const uint4*>(smem + rd_nw_off(H));
  cp_async_wait(0);
  __syncthreads();
  for (int i = tid; i < H / 8; i += NT) {
    const uint4 v = rms_apply8(hg[i], nw[i], rs);
    xs[i] = v;
    if (blockIdx.x == 0) reinterpret_cast<uint4*>(a.xn_out)[i] = v;
  }
  cp_async_wait(0);
  __syncthreads();
  if (warp < ne) {
    const float v = router_logit8(reinterpret_cast<const __nv_bfloat162*>(xs),
                                  reinterpret_cast<const uint32_t*>(wq + (size_t)warp * H),
                                  ws + warp * gpr, wb + warp * gpr, H);
    if (lane == 0) a.lg_ws[e0 + warp] = v;
  }
  __syncthreads();  // this CTA's logits are stored before thread 0 releases them
  if (tid == 0) *flag = atom_add_acq_rel_gpu(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();  // the last CTA: every CTA's logits, acquired by thread 0, are visible
  if (!*flag) return;
  if (tid < 32) slot[tid] = -1;
  if (warp == 0) topk_scores_warp([&](int e) { return __ldcg(a.lg_ws + e); }, E, ebs,
                                  a.score_fn, keys, vals);
  __syncthreads();
  topk_rank(keys, E, a.k, slot, tid, NT);
  __syncthreads();
  if (warp == 0) {
    int idx = -1;
    float wt = 0.f;
    topk_pick_warp(vals, slot, a.k, a.norm, &idx, &wt, nullptr);
    if (lane < a.k) {
      a.inds[lane] = idx;
      a.wout[lane] = __float2bfloat16_rn(wt);
    }
    if (a.logits)
      for (int e = lane; e < E; e += 32) a.logits[e] = __ldcg(a.lg_ws + e);
  }
  if (tid == 0) *a.counter = 0u;  // ready for the next call
}

// ---- MoE experts for one token ---------------------------------------------------------------

struct MdArgs {
  const __nv_bfloat16* xn;  // [H] normalised token
  const int32_t* inds;      // [k]
  const __nv_bfloat16* w;   // [k]
  int H, I, I_sh, E, k, Imax;
  float routed_scale;
  const uint32_t *g_q, *u_q, *d_q;
  const __nv_bfloat16 *g_s, *g_b, *u_s, *u_b, *d_s, *d_b;
  const uint32_t *sg_q, *su_q, *sd_q;
  const __nv_bfloat16 *sg_s, *sg_b, *su_s, *su_b, *sd_s, *sd_b;
  __nv_bfloat16* hbuf;       // [k + 1, Imax] SwiGLU outputs
  const __nv_bfloat16* res;  // [H] residual, or null
  __nv_bfloat16* out;        // [H]
  float* ypart;              // [H/16][k + 1][16] per-group down outputs (bf16-valued)
  unsigned int* counters;    // [H/16] groups done per 16-row slice (zero between calls)
};

// Workspace of lg_moe_decode: counters (a fixed 4 KiB block, one per 16-row slice for any H up
// to 16,384, so calls of different sizes sharing one workspace never overlap them with data) |
// per-group outputs [ceil(H/16)][k+1][16] fp32 | SwiGLU outputs [k+1][Imax] bf16.
constexpr size_t MD_CTRL_BYTES = 4096;
struct MdWs {
  size_t counters, ypart, hbuf, total;
};
__host__ __device__ __forceinline__ MdWs md_ws(int H, int Imax, int k) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t nt = (H + 15) / 16, G = k + 1;
  MdWs w;
  w.counters = 0;
  w.ypart = MD_CTRL_BYTES;
  w.hbuf = w.ypart + up(4 * nt * G * 16);
  w.total = w.hbuf + up(2 * G * (size_t)Imax);
  return w;
}

constexpr int GU_WARPS = 8;
constexpr int DN_WARPS = 4;

// grid (Imax/16, k + 1): group j < k is pick j, group k the shared expert. Shared memory as
// dgemv_kernel's with a two-tile (gate, up) stage.
template <int V>
__global__ void __launch_bounds__(GU_WARPS * 32, 4) moe_dec_gateup_kernel(MdArgs a) {
  constexpr int NW = GU_WARPS;
  extern __shared__ __align__(128) uint8_t smem[];
  const int H = a.H, gpr = H / 64;
  float* red = reinterpret_cast<float*>(smem + 32);  // [2][NW][16]
  uint4* xs = reinterpret_cast<uint4*>(smem + ((32u + 2u * 2u * NW * 16u * 4u + 15u) & ~15u));
  float* gsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + 2 * H);
  uint8_t* ring = smem + dg_ring_off(H, NW);
  const uint32_t pitch = tile_pitch(H), tb = tile_bytes(H);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = lane >> 2, c4 = lane & 3;
  const int j = blockIdx.y;
  const bool sh = (j == a.k);
  const int Ig = sh ? a.I_sh : a.I;
  const int m0 = blockIdx.x * 16;
  const int rows = min(16, Ig - m0);
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t slim = dyn_smem_bytes();
  const uint32_t *gq = a.sg_q, *uq = a.su_q;
  const __nv_bfloat16 *gs = a.sg_s, *gb = a.sg_b, *us = a.su_s, *ub = a.su_b;
  // the weight tiles come by bulk copies (issued by one thread) that complete on this barrier
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* berr = reinterpret_cast<int*>(smem + 8);
  if (tid == 0) {
    *berr = 0;
    mbar_init(bar, 1);
    fence_mbar_init();
    if (sh && rows == 16) {  // the shared expert is static: stream it before the wait
      mbar_arrive_expect_tx(bar, 2u * tile_bulk_bytes(H));
      tile_load_bulk(ring, gq, gs, gb, m0, H, bar);
      tile_load_bulk(ring + tb, uq, us, ub, m0, H, bar);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (rows <= 0) return;
  // the normalised token (the router's output): its copy overlaps the read of the pick
  const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(a.xn);
  for (int c = tid; c < H / 8; c += NW * 32)
    cp_async16(reinterpret_cast<uint8_t*>(xs) + c * 16, xsrc + (size_t)c * 16, pol, smem, slim);
  cp_async_commit();
  if (!sh) {
    const int e = a.inds[j];
    if (e < 0 || e >= a.E) {  // no expert: the down kernel skips this pick
      cp_async_wait(0);  // leave no copy in flight behind
      return;
    }
    const size_t wo = (size_t)e * a.I * (H / 8), so = (size_t)e * a.I * gpr;
    gq = a.g_q + wo; gs = a.g_s + so; gb = a.g_b + so;
    uq = a.u_q + wo; us = a.u_s + so; ub = a.u_b + so;
    if (tid == 0) {
      mbar_arrive_expect_tx(bar, 2u * tile_bulk_bytes(H));
      tile_load_bulk(ring, gq, gs, gb, m0, H, bar);
      tile_load_bulk(ring + tb, uq, us, ub, m0, H, bar);
    }
  }
  cp_async_wait(0);  // the activations
  __syncthreads();
  group_sums(xs, gpr, gsum);
  const int gpw = (gpr + NW - 1) / NW;
  const int gw0 = warp * gpw, gwn = max(0, min(gpr, gw0 + gpw) - gw0);
  if (!__syncthreads_and(mbar_wait(bar, 0, berr, 1, 400000000LL))) {  // CTA-uniform exit
    // the tiles never arrived: record it, let the copies drain (bounded), leave the rows unset
    if (tid == 0 && atomicCAS(&g_stage_check[0], 0ull, 4ull) == 0ull) g_stage_check[3] = 0xB1u;
    for (const long long t0 = clock64(); !mbar_try_wait(bar, 0) && clock64() - t0 < 400000000LL;) {
    }
    return;
  }
  __syncthreads();
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const uint8_t* tile = ring + m * tb;
    const SbRows sr = sb_rows(tile, H, rows, m0, Ig, m ? us : gs, m ? ub : gb, r);
    float y0 = 0.f, y8 = 0.f;
    warp_tile_dot<V>(y0, y8, tile, pitch, sr.s0, sr.s8, sr.b0, sr.b8, gw0, gwn, xs, gsum, r, c4);
    if (c4 == 0) {
      red[(m * NW + warp) * 16 + r] = y0;
      red[(m * NW + warp) * 16 + r + 8] = y8;
    }
  }
  __syncthreads();
  float* red2 = red + 2 * NW * 16;  // [2][16]
  if (tid < 32) {  // (mat, row): sum over the warps
    const int m = tid >> 4, rr = tid & 15;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red[(m * NW + w) * 16 + rr];
    red2[tid] = v;
  }
  __syncthreads();
  if (tid < rows) a.hbuf[(size_t)j * a.Imax + m0 + tid] = swiglu_mlx(red2[tid], red2[16 + tid]);
}

// grid (ceil(H/16), k + 1): one 16-row slice of the hidden dimension for one group (pick j < k,
// the shared expert j = k). The CTA is small, so it becomes resident beside the gate/up CTAs
// and streams its weight tile before its wait (the picks come from the router, two kernels
// back). Each CTA writes its group's bf16-rounded outputs; the last CTA of a slice to finish
// combines the groups in fixed order (fp32, one rounding) and adds the residual.
template <int V>
__global__ void __launch_bounds__(DN_WARPS * 32) moe_dec_down_kernel(MdArgs a) {
  constexpr int NW = DN_WARPS, NT = NW * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int G = a.k + 1, Imax = a.Imax, H = a.H;
  float* red = reinterpret_cast<float*>(smem);      // [NW][16]
  float* cw = red + NW * 16;                        // [G] combine weights (last CTA)
  int* ce = reinterpret_cast<int*>(cw + 33);        // [G] picks (last CTA)
  int* flag = ce + 33;
  uint4* hs = reinterpret_cast<uint4*>(smem + 1024);                  // [Imax/8]
  float* gsum = reinterpret_cast<float*>(smem + 1024 + 2 * Imax);     // [Imax/64]
  uint8_t* tile = smem + ((1024 + 2 * Imax + 4 * (Imax / 64) + 127) & ~127);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = lane >> 2, c4 = lane & 3;
  const int mt = blockIdx.x, j = blockIdx.y;
  const int m0 = mt * 16;
  const int rows = min(16, H - m0);
  (void)lane;
  // The picks come from the router, two kernels back, and the residual from the attention
  // output projection, three back: both have completed (the kernel in between waited for its
  // predecessor before letting this one start), so they are read before the wait (L2 loads).
  int e;
  if (j < a.k) {
    e = __ldcg(a.inds + j);
    if (e < 0 || e >= a.E) e = -1;
  } else {
    e = a.I_sh > 0 ? -2 : -1;  // -2: the shared expert; -1: no expert
  }
  float resv = 0.f;
  if (a.res && tid < rows) resv = bf2f(__ldcg(a.res + m0 + tid));
  const int Kj = e == -2 ? a.I_sh : a.I, gpr = Kj / 64;
  const __nv_bfloat16* sg = e == -2 ? a.sd_s : a.d_s + (size_t)(e < 0 ? 0 : e) * H * (a.I / 64);
  const __nv_bfloat16* bg = e == -2 ? a.sd_b : a.d_b + (size_t)(e < 0 ? 0 : e) * H * (a.I / 64);
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t slim = dyn_smem_bytes();
  if (e != -1) {
    const uint32_t* dq = e == -2 ? a.sd_q : a.d_q + (size_t)e * H * (a.I / 8);
    tile_load(tile, dq, sg, bg, m0, rows, Kj, pol, smem, slim);
  }
  cp_async_commit();
  pdl_wait();
  pdl_trigger();
  float y[2] = {0.f, 0.f};
  if (e != -1) {
    // this group's SwiGLU outputs (the previous kernel's output; every slice reads them)
    const uint64_t pol_keep = l2_evict_normal_policy();
    const uint8_t* hsrc = reinterpret_cast<const uint8_t*>(a.hbuf + (size_t)j * Imax);
    for (int c = tid; c < Kj / 8; c += NT)
      cp_async16(reinterpret_cast<uint8_t*>(hs) + c * 16, hsrc + (size_t)c * 16, pol_keep, smem,
                 slim);
    cp_async_commit();
    cp_async_wait(0);
    __syncthreads();
    group_sums(hs, gpr, gsum);
    __syncthreads();
    const int gpw = (gpr + NW - 1) / NW;
    const int gw0 = warp * gpw, gwn = max(0, min(gpr, gw0 + gpw) - gw0);
    const SbRows sr = sb_rows(tile, Kj, rows, m0, H, sg, bg, r);
    float y0 = 0.f, y8 = 0.f;
    warp_tile_dot<V>(y0, y8, tile, tile_pitch(Kj), sr.s0, sr.s8, sr.b0, sr.b8, gw0, gwn, hs,
                     gsum, r, c4);
    if (c4 == 0) {
      red[warp * 16 + r] = y0;
      red[warp * 16 + r + 8] = y8;
    }
    __syncthreads();
    if (tid < 16) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) v += red[w * 16 + tid];
      y[0] = round_bf16(v);  // gather_qmm / quantized_matmul output
    }
  }
  if (tid < 16) a.ypart[((size_t)mt * G + j) * 16 + tid] = y[0];
  __syncthreads();  // the group's partial is stored before thread 0 releases it
  if (tid == 0) *flag = atom_add_acq_rel_gpu(a.counters + mt, 1u) == (unsigned)(G - 1);
  __syncthreads();  // the last group: every group's partial, acquired by thread 0, is visible
  if (!*flag) return;
  // the last group of this slice: combine every group in order
  if (tid < G) {
    int ej;
    float wj = 1.0f;
    if (tid < a.k) {
      ej = __ldcg(a.inds + tid);
      if (ej < 0 || ej >= a.E) ej = -1;
      wj = bf2f(__ldcg(a.w + tid)) * a.routed_scale;
    } else {
      ej = a.I_sh > 0 ? -2 : -1;
    }
    ce[tid] = ej;
    cw[tid] = wj;
  }
  __syncthreads();
  if (tid < rows) {
    float acc = 0.f;
    for (int g = 0; g < G; ++g)
      if (ce[g] != -1)
        acc = __fadd_rn(acc, __fmul_rn(cw[g], __ldcg(a.ypart + ((size_t)mt * G + g) * 16 + tid)));
    float o = round_bf16(acc);
    if (a.res) o = __fadd_rn(o, resv);
    a.out[m0 + tid] = __float2bfloat16_rn(o);
  }
  if (tid == 0) a.counters[mt] = 0u;  // ready for the next call
}

__host__ __device__ __forceinline__ uint32_t md_down_smem(int Imax) {
  return ((1024 + 2 * Imax + 4 * (Imax / 64) + 127) & ~127) + tile_bytes(Imax);
}

// ---- host side -------------------------------------------------------------------------------

static constexpr size_t SMEM_CAP = 227 * 1024;

// Raise a kernel's dynamic shared memory limit once per device (to the cap, so later calls
// with other sizes need nothing).
template <typename Kern>
static cudaError_t allow_smem(Kern k, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(k));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_CAP);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

// scale-vector width for a warp's share of gpr groups over nw warps
static int vec_width(int gpr, int nw) {
  if (gpr % nw) return 1;
  const int gpw = gpr / nw;
  return gpw % 8 == 0 ? 8 : gpw % 4 == 0 ? 4 : gpw % 2 == 0 ? 2 : 1;
}

template <bool GLU, int NW, int V>
static cudaError_t launch_dgemv_v(const DgArgs& a, const PrepArgs& p, dim3 grid, size_t smem,
                                  cudaStream_t st) {
  if constexpr (!GLU && NW == 8) {
    if (a.prep) {
      cudaError_t e = allow_smem(dgemv_prep_kernel<V>, smem);
      return e != cudaSuccess
                 ? e
                 : launch_k(dgemv_prep_kernel<V>, grid, dim3(NW * 32), smem, st, a, p);
    }
  }
  cudaError_t e = allow_smem(dgemv_kernel<GLU, NW, V>, smem);
  return e != cudaSuccess ? e
                          : launch_k(dgemv_kernel<GLU, NW, V>, grid, dim3(NW * 32), smem, st, a);
}

template <bool GLU, int NW>
static cudaError_t launch_dgemv_nw(const DgArgs& a, const PrepArgs& p, dim3 grid, size_t smem,
                                   cudaStream_t st) {
  switch (vec_width(a.K / 64, NW)) {
    case 8: return launch_dgemv_v<GLU, NW, 8>(a, p, grid, smem, st);
    case 4: return launch_dgemv_v<GLU, NW, 4>(a, p, grid, smem, st);
    case 2: return launch_dgemv_v<GLU, NW, 2>(a, p, grid, smem, st);
    default: return launch_dgemv_v<GLU, NW, 1>(a, p, grid, smem, st);
  }
}

// warps per dense-GEMV CTA: 16 for long rows, else 8
static int dg_warps(int K) { return K / 64 >= 64 ? 16 : 8; }

template <bool GLU>
static cudaError_t launch_dgemv(const DgArgs& a, const PrepArgs& p, dim3 grid, size_t smem,
                                cudaStream_t st) {
  return dg_warps(a.K) == 16 ? launch_dgemv_nw<GLU, 16>(a, p, grid, smem, st)
                             : launch_dgemv_nw<GLU, 8>(a, p, grid, smem, st);
}

static int check_tile_mat(const void* q, const void* s, const void* b, const char* what) {
  if (!q || !s || !b) return fail(LG_ERR_INVALID, "%s: NULL weight/scales/biases", what);
  if (!aligned(q, 16) || !aligned(s, 16) || !aligned(b, 16))
    return fail(LG_ERR_INVALID, "%s: weights, scales and biases must be 16-byte aligned", what);
  return LG_OK;
}

}  // namespace lg

using namespace lg;

// Tile plan and launch of the dense decode GEMV. one_tile: fail unless every CTA gets exactly
// one tile (the fused prologue needs it).
static int dgemv_launch(DgArgs& a, const PrepArgs& p, bool glu, bool one_tile,
                        cudaStream_t st) {
  const int NM = glu ? 2 : 1, K = a.K;
  a.tiles = (a.N + 15) / 16;
  const size_t stage = (size_t)NM * tile_bytes(K), fixed = dg_ring_off(K, dg_warps(K));
  const int sms = device_sm_count();
  // one tile per CTA while all of them fit on the GPU at once, else a ring of tiles per CTA
  const int per_sm = (int)((200 * 1024) / (fixed + stage));
  int grid, stages;
  if (per_sm >= 1 && a.tiles <= per_sm * sms) {
    grid = a.tiles;
    stages = 1;
  } else {
    if (one_tile)
      return fail(LG_ERR_UNSUPPORTED, "decode_gemv: %d tiles do not fit one per CTA", a.tiles);
    grid = 2 * sms;
    const long long room = 96 * 1024 - (long long)fixed;
    stages = room > 0 ? (int)(room / (long long)stage) : 1;
    stages = stages < 1 ? 1 : stages > DG_MAX_STAGES ? DG_MAX_STAGES : stages;
    const int need = (a.tiles + grid - 1) / grid;
    if (stages > need) stages = need;
  }
  a.stages = stages;
  const size_t smem = fixed + stages * stage;
  LG_CHECK_ARG(smem <= SMEM_CAP, "decode_gemv: K=%d needs %zu bytes of shared memory", K, smem);
  prof_begin("decode_gemv", st);
  LG_CUDA_TRY(glu ? launch_dgemv<true>(a, p, dim3(grid), smem, st)
                  : launch_dgemv<false>(a, p, dim3(grid), smem, st));
  prof_end("decode_gemv", st);
  LG_LAUNCH_CHECK("dgemv");
  return LG_OK;
}

extern "C" int lg_decode_gemv(const void* x, int K, int N, const uint32_t* w_q, const void* w_s,
                              const void* w_b, const uint32_t* u_q, const void* u_s,
                              const void* u_b, const void* norm_w, float eps,
                              const void* residual, void* out, void* stream) {
  LG_CHECK_ARG(K > 0 && K % 64 == 0 && N > 0, "decode_gemv: need K %% 64 == 0 (K=%d, N=%d)", K,
               N);
  LG_CHECK_ARG(K <= 16384, "decode_gemv: K=%d > 16384", K);
  LG_CHECK_ARG(x && out, "decode_gemv: NULL pointer");
  LG_CHECK_ARG(aligned(x, 16) && (!norm_w || aligned(norm_w, 16)),
               "decode_gemv: x and the norm weight must be 16-byte aligned");
  int rc = check_tile_mat(w_q, w_s, w_b, "decode_gemv");
  if (rc) return rc;
  const bool glu = u_q != nullptr;
  if (glu) {
    if ((rc = check_tile_mat(u_q, u_s, u_b, "decode_gemv (up)"))) return rc;
    LG_CHECK_ARG(!residual, "decode_gemv: no residual with a gate/up pair");
  }
  DgArgs a = {};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.q[0] = w_q;
  a.s[0] = static_cast<const __nv_bfloat16*>(w_s);
  a.b[0] = static_cast<const __nv_bfloat16*>(w_b);
  a.q[1] = u_q;
  a.s[1] = static_cast<const __nv_bfloat16*>(u_s);
  a.b[1] = static_cast<const __nv_bfloat16*>(u_b);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.K = K;
  a.N = N;
  a.prep = 0;
  return dgemv_launch(a, PrepArgs{}, glu, false, static_cast<cudaStream_t>(stream));
}

extern "C" size_t lg_decode_qkv_prep_workspace_bytes(int Hq, int Hkv) {
  return align_up(4 * (size_t)(Hq > 0 && Hkv > 0 ? Hq + 2 * Hkv : 0), 256);
}

extern "C" int lg_decode_qkv_prep(const void* x, int K, const uint32_t* w_q, const void* w_s,
                                  const void* w_b, const void* norm_w, float eps, int Hq,
                                  int Hkv, int D, const void* qn_w, const void* kn_w,
                                  float qk_eps, float rope_theta, const int32_t* pos_dev,
                                  int pos_host, int gate_per_head, void* qkvg_out, void* q_out,
                                  void* gate_out, void* k_cache, void* v_cache, uint32_t* k_q,
                                  void* k_s, void* k_b, uint32_t* v_q, void* v_s, void* v_b,
                                  int cap, const float* inv_freq, int rot_dims, float mscale,
                                  int ring, int row0, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  LG_CHECK_ARG(K > 0 && K % 64 == 0 && K <= 16384, "decode_qkv_prep: hidden %d", K);
  LG_CHECK_ARG(Hq > 0 && Hkv > 0 && D % 64 == 0 && D <= 256,
               "decode_qkv_prep: heads %d/%d, head_dim %d (a multiple of 64, <= 256)", Hq, Hkv, D);
  LG_CHECK_ARG(x && norm_w && qn_w && kn_w && qkvg_out && q_out && gate_out,
               "decode_qkv_prep: NULL pointer");
  LG_CHECK_ARG(2 * K >= D, "decode_qkv_prep: hidden %d below half of head_dim %d", K, D);
  if (dg_warps(K) != 8)  // the fused form is built for 8-warp CTAs (hidden < 4096)
    return fail(LG_ERR_UNSUPPORTED, "decode_qkv_prep: hidden %d takes the two-launch form", K);
  const bool q8 = k_q != nullptr;
  LG_CHECK_ARG(q8 ? (k_s && k_b && v_q && v_s && v_b && !k_cache && !v_cache)
                  : (k_cache && v_cache),
               "decode_qkv_prep: give either the bf16 cache or the 8-bit cache");
  LG_CHECK_ARG(aligned(x, 16) && aligned(norm_w, 16),
               "decode_qkv_prep: x and the norm weight must be 16-byte aligned");
  LG_CHECK_ARG(pos_dev || ring > 0 || (pos_host - row0 >= 0 && pos_host - row0 < cap),
               "decode_qkv_prep: position %d beyond the cache rows %d..%d", pos_host, row0,
               row0 + cap - 1);
  LG_CHECK_ARG(ring == 0 || ring == cap, "decode_qkv_prep: a ring buffer has %d rows, not %d",
               cap, ring);
  int rc = check_tile_mat(w_q, w_s, w_b, "decode_qkv_prep");
  if (rc) return rc;
  const size_t need = lg_decode_qkv_prep_workspace_bytes(Hq, Hkv);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "decode_qkv_prep: workspace needs %zu zeroed bytes", need);
  DgArgs a = {};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.q[0] = w_q;
  a.s[0] = static_cast<const __nv_bfloat16*>(w_s);
  a.b[0] = static_cast<const __nv_bfloat16*>(w_b);
  a.out = static_cast<__nv_bfloat16*>(qkvg_out);
  a.K = K;
  a.N = (Hq + 2 * Hkv) * D + (gate_per_head ? Hq : Hq * D);
  a.prep = 1;
  a.head_cnt = static_cast<unsigned int*>(workspace);
  PrepArgs p = {};
  if (int rc2 = prep_extend(&p, D, inv_freq, rot_dims, mscale, ring, row0, "decode_qkv_prep"))
    return rc2;
  p.qkvg = static_cast<const __nv_bfloat16*>(qkvg_out);
  p.qn_w = static_cast<const __nv_bfloat16*>(qn_w);
  p.kn_w = static_cast<const __nv_bfloat16*>(kn_w);
  p.pos_dev = pos_dev;
  p.pos_host = pos_host;
  p.T = 1;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.cap = cap;
  p.gate_per_head = gate_per_head;
  p.eps = qk_eps;
  p.log2_theta = log2f(rope_theta);
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.gate_out = static_cast<__nv_bfloat16*>(gate_out);
  p.kq = k_q;
  p.ks = static_cast<__nv_bfloat16*>(k_s);
  p.kb = static_cast<__nv_bfloat16*>(k_b);
  p.vq = v_q;
  p.vs = static_cast<__nv_bfloat16*>(v_s);
  p.vb = static_cast<__nv_bfloat16*>(v_b);
  return dgemv_launch(a, p, false, true, static_cast<cudaStream_t>(stream));
}

extern "C" int lg_router_decode_supported(int H, int E) {
  // every CTA's slice of the scales must be whole 16-byte chunks
  return H > 0 && H % 64 == 0 && H <= 16384 && E > 0 && E <= 256 &&
         ((H / 64) % 8 == 0 || E % RD_WARPS == 0) && rd_smem(H) <= SMEM_CAP;
}

extern "C" size_t lg_router_decode_workspace_bytes(int E) {
  return align_up(16 + 4 * (size_t)(E > 0 ? E : 0), 256);
}

extern "C" int lg_router_decode(const void* h, const void* norm_w, float eps, int H,
                                const uint32_t* gate_q, const void* gate_s, const void* gate_b,
                                const float* e_bias, int E, int k, int norm_topk_prob,
                                int score_fn, void* xn_out, int32_t* inds, void* weights,
                                float* logits, void* workspace, size_t workspace_bytes,
                                void* stream) {
  LG_CHECK_ARG(H > 0 && H % 64 == 0 && H <= 16384, "router_decode: hidden %d", H);
  LG_CHECK_ARG(E > 0 && E <= 256, "router_decode: E=%d not in [1, 256]", E);
  LG_CHECK_ARG(k >= 1 && k <= E && k <= 32, "router_decode: k=%d must be in [1, min(E, 32)]", k);
  LG_CHECK_ARG(score_fn == LG_SCORE_SIGMOID || score_fn == LG_SCORE_SOFTMAX,
               "router_decode: score_fn %d", score_fn);
  LG_CHECK_ARG(h && norm_w && gate_q && gate_s && gate_b && xn_out && inds && weights,
               "router_decode: NULL pointer");
  LG_CHECK_ARG(aligned(h, 16) && aligned(norm_w, 16) && aligned(xn_out, 16) &&
                   aligned(gate_q, 16) && aligned(gate_s, 16) && aligned(gate_b, 16),
               "router_decode: operands must be 16-byte aligned");
  if (!lg_router_decode_supported(H, E))
    return fail(LG_ERR_UNSUPPORTED, "router_decode: E=%d x H=%d is not supported", E, H);
  const size_t need = lg_router_decode_workspace_bytes(E);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "router_decode: workspace needs %zu bytes (256-aligned; its "
                "first 16 bytes zero)", need);
  RdArgs a;
  a.h = static_cast<const __nv_bfloat16*>(h);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.gq = gate_q;
  a.gs = static_cast<const __nv_bfloat16*>(gate_s);
  a.gb = static_cast<const __nv_bfloat16*>(gate_b);
  a.ebias = e_bias;
  a.H = H;
  a.E = E;
  a.k = k;
  a.norm = norm_topk_prob;
  a.score_fn = score_fn;
  a.xn_out = static_cast<__nv_bfloat16*>(xn_out);
  a.inds = inds;
  a.wout = static_cast<__nv_bfloat16*>(weights);
  a.logits = logits;
  a.counter = static_cast<unsigned int*>(workspace);
  a.lg_ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + 16);
  const size_t smem = rd_smem(H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LG_CUDA_TRY(allow_smem(router_decode_kernel, smem));
  prof_begin("router_decode", st);
  LG_CUDA_TRY(launch_k(router_decode_kernel, dim3((E + RD_WARPS - 1) / RD_WARPS),
                       dim3(RD_WARPS * 32), smem, st, a));
  prof_end("router_decode", st);
  LG_LAUNCH_CHECK("router_decode");
  return LG_OK;
}


extern "C" size_t lg_moe_decode_workspace_bytes(int H, int I, int I_shared, int k) {
  const int Imax = I > I_shared ? I : I_shared;
  return md_ws(H > 0 ? H : 0, Imax, k > 0 ? k : 0).total;
}

extern "C" int lg_moe_decode_supported(int H, int I, int I_shared, int k) {
  if (H <= 0 || H % 64 || H > 16384 || I <= 0 || I % 64 || I_shared < 0 || I_shared % 64 ||
      k < 1 || k > 32)
    return 0;
  const int Imax = I > I_shared ? I : I_shared;
  return md_down_smem(Imax) <= SMEM_CAP &&
         dg_ring_off(H, GU_WARPS) + 2 * (size_t)tile_bytes(H) <= SMEM_CAP;
}

template <int V>
static cudaError_t launch_moe_gateup(const MdArgs& a, dim3 g, size_t smem, cudaStream_t st) {
  cudaError_t e = allow_smem(moe_dec_gateup_kernel<V>, smem);
  return e != cudaSuccess
             ? e
             : launch_k(moe_dec_gateup_kernel<V>, g, dim3(GU_WARPS * 32), smem, st, a);
}

template <int V>
static cudaError_t launch_moe_down(const MdArgs& a, dim3 g, size_t smem, cudaStream_t st) {
  cudaError_t e = allow_smem(moe_dec_down_kernel<V>, smem);
  return e != cudaSuccess
             ? e
             : launch_k(moe_dec_down_kernel<V>, g, dim3(DN_WARPS * 32), smem, st, a);
}

extern "C" int lg_moe_decode(const void* xn, const int32_t* inds, const void* weights, int H,
                             int I, int E, int k, float routed_scale, const uint32_t* g_q,
                             const void* g_s, const void* g_b, const uint32_t* u_q,
                             const void* u_s, const void* u_b, const uint32_t* d_q,
                             const void* d_s, const void* d_b, int I_shared,
                             const uint32_t* sg_q, const void* sg_s, const void* sg_b,
                             const uint32_t* su_q, const void* su_s, const void* su_b,
                             const uint32_t* sd_q, const void* sd_s, const void* sd_b,
                             const void* residual, void* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  LG_CHECK_ARG(H > 0 && H % 64 == 0 && H <= 16384, "moe_decode: hidden %d", H);
  LG_CHECK_ARG(E > 0 && k >= 1 && k <= E && k <= 32 && I > 0 && I % 64 == 0,
               "moe_decode: E=%d k=%d I=%d (I %% 64 == 0)", E, k, I);
  LG_CHECK_ARG(I_shared >= 0 && I_shared % 64 == 0, "moe_decode: shared intermediate %d",
               I_shared);
  LG_CHECK_ARG(xn && inds && weights && out, "moe_decode: NULL pointer");
  LG_CHECK_ARG(aligned(xn, 16) && (!residual || aligned(residual, 2)),
               "moe_decode: xn must be 16-byte aligned");
  int rc;
  if ((rc = check_tile_mat(g_q, g_s, g_b, "moe_decode gate")) ||
      (rc = check_tile_mat(u_q, u_s, u_b, "moe_decode up")) ||
      (rc = check_tile_mat(d_q, d_s, d_b, "moe_decode down")))
    return rc;
  if (I_shared &&
      ((rc = check_tile_mat(sg_q, sg_s, sg_b, "moe_decode shared gate")) ||
       (rc = check_tile_mat(su_q, su_s, su_b, "moe_decode shared up")) ||
       (rc = check_tile_mat(sd_q, sd_s, sd_b, "moe_decode shared down"))))
    return rc;
  const size_t need = lg_moe_decode_workspace_bytes(H, I, I_shared, k);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(LG_ERR_WORKSPACE, "moe_decode: workspace needs %zu bytes (256-aligned, the "
                "first %zu zero)", need, MD_CTRL_BYTES);
  if (!lg_moe_decode_supported(H, I, I_shared, k))
    return fail(LG_ERR_UNSUPPORTED, "moe_decode: k=%d I=%d/%d H=%d exceed the shared memory", k,
                I, I_shared, H);
  const int Imax = I > I_shared ? I : I_shared;
  const MdWs W = md_ws(H, Imax, k);
  MdArgs a;
  a.xn = static_cast<const __nv_bfloat16*>(xn);
  a.inds = inds;
  a.w = static_cast<const __nv_bfloat16*>(weights);
  a.H = H;
  a.I = I;
  a.I_sh = I_shared;
  a.E = E;
  a.k = k;
  a.Imax = Imax;
  a.routed_scale = routed_scale;
  a.g_q = g_q; a.u_q = u_q; a.d_q = d_q;
  a.g_s = static_cast<const __nv_bfloat16*>(g_s);
  a.g_b = static_cast<const __nv_bfloat16*>(g_b);
  a.u_s = static_cast<const __nv_bfloat16*>(u_s);
  a.u_b = static_cast<const __nv_bfloat16*>(u_b);
  a.d_s = static_cast<const __nv_bfloat16*>(d_s);
  a.d_b = static_cast<const __nv_bfloat16*>(d_b);
  a.sg_q = sg_q; a.su_q = su_q; a.sd_q = sd_q;
  a.sg_s = static_cast<const __nv_bfloat16*>(sg_s);
  a.sg_b = static_cast<const __nv_bfloat16*>(sg_b);
  a.su_s = static_cast<const __nv_bfloat16*>(su_s);
  a.su_b = static_cast<const __nv_bfloat16*>(su_b);
  a.sd_s = static_cast<const __nv_bfloat16*>(sd_s);
  a.sd_b = static_cast<const __nv_bfloat16*>(sd_b);
  char* wsb = static_cast<char*>(workspace);
  a.counters = reinterpret_cast<unsigned int*>(wsb + W.counters);
  a.ypart = reinterpret_cast<float*>(wsb + W.ypart);
  a.hbuf = reinterpret_cast<__nv_bfloat16*>(wsb + W.hbuf);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.out = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem_gu = dg_ring_off(H, GU_WARPS) + 2 * (size_t)tile_bytes(H);
  const int Vg = vec_width(H / 64, GU_WARPS);
  const int vi = vec_width(I / 64, DN_WARPS), vs = I_shared ? vec_width(I_shared / 64, DN_WARPS) : vi;
  const int Vd = vi < vs ? vi : vs;
  dim3 g1((Imax + 15) / 16, k + 1), g2((H + 15) / 16, k + 1);
  const size_t smem_dn = md_down_smem(Imax);
  prof_begin("moe_decode", st);
  LG_CUDA_TRY(Vg == 8   ? launch_moe_gateup<8>(a, g1, smem_gu, st)
              : Vg == 4 ? launch_moe_gateup<4>(a, g1, smem_gu, st)
              : Vg == 2 ? launch_moe_gateup<2>(a, g1, smem_gu, st)
                        : launch_moe_gateup<1>(a, g1, smem_gu, st));
  LG_LAUNCH_CHECK("moe_dec_gateup");
  LG_CUDA_TRY(Vd == 8   ? launch_moe_down<8>(a, g2, smem_dn, st)
              : Vd == 4 ? launch_moe_down<4>(a, g2, smem_dn, st)
              : Vd == 2 ? launch_moe_down<2>(a, g2, smem_dn, st)
                        : launch_moe_down<1>(a, g2, smem_dn, st));
  prof_end("moe_decode", st);
  LG_LAUNCH_CHECK("moe_dec_down");
  return LG_OK;
}

extern "C" int lg_decode_status(unsigned long long* check, int reset) {
  LG_CHECK_ARG(check, "decode_status: NULL pointer");
  LG_CUDA_TRY(cudaMemcpyFromSymbol(check, g_stage_check, sizeof(g_stage_check)));
  if (reset) {
    const unsigned long long zero[4] = {0, 0, 0, 0};
    LG_CUDA_TRY(cudaMemcpyToSymbol(g_stage_check, zero, sizeof(g_stage_check)));
  }
  return LG_OK;
}
