// Decode-size MoE expert products: split-K GEMV on the tensor cores (mma.sync m16n8k16 bf16).
//
// Few picks per expert make these products HBM-bound: each weight byte is read once and the
// work per byte is small, so the kernels are built around 8-byte-per-lane streaming loads of
// the MLX 4-bit words and keep the arithmetic off the FP32 pipe:
//  * a 4-bit code c becomes the exact bf16 value c via (0x4300 | c) - 128 (two codes per
//    32-bit register, one LOP3 + one packed subtract);
//  * the K order inside each 16-wide MMA k-block is permuted so that one 32-bit weight word
//    feeds a thread's whole A fragment for two k-blocks; the activations use the same order;
//  * the affine dequantisation is applied per 64-group after the MMA:
//      y[r] = sum_g scale[r,g] * (sum_{k in g} code[r,k] x[k]) + bias[r,g] * sum_{k in g} x[k]
//    which equals dot(x, scale * code + bias) (laguna_mlx/q8_attn.py:50 form).
//
// gate/up kernel: one CTA = 4 warps = one 16-row tile of the intermediate dimension for one
//   expert group (gate rows and up rows), split-K over the 4 warps, SwiGLU in the epilogue with
//   the bf16 rounding points of the MLX graph (laguna.py:122): g, u -> bf16; silu = g*sigmoid(g)
//   with each op rounded to bf16; h = bf16(silu * u).
// down kernel: one CTA = one 16-row tile of the hidden dimension for one expert group, split-K
//   over 4 warps; the epilogue rounds y to bf16 (gather_qmm output) and stores it per pick
//   row (routed picks, then the shared expert's rows); the weighted combine of
//   laguna.py:149-150 is a separate fixed-order pass over those rows.
#include "common.cuh"
#include "decode_core.cuh"
#include "gemv_core.cuh"
#include "moe.cuh"

namespace lg {

// token (activation row) of group row j: routed picks p < P come from token p / k, shared
// rows p >= P from token p - P.
__device__ __forceinline__ int row_token(int p, int P, int k) { return p < P ? p / k : p - P; }

constexpr int GV_WARPS = 4;
// dynamic shared memory: [0, 128) mbarrier and wait flag, then the cross-warp reduction, then
// (staged kernels) the weight tile(s) in the padded layout of decode_core.cuh
constexpr uint32_t GV_HDR = 128;
constexpr uint32_t GV_RED_GU = GV_WARPS * 2 * 32 * 4 * 4;
constexpr uint32_t GV_RED_DN = GV_WARPS * 32 * 4 * 4;
constexpr long long GV_WAIT_CYCLES = 400000000LL;  // ~0.2 s: the tile copies are long done

static uint32_t gv_smem_gu(int H, bool staged) {
  return GV_HDR + GV_RED_GU + (staged ? 2 * tile_bytes(H) : 0);
}
static uint32_t gv_smem_dn(int Kmax, bool staged) {
  return GV_HDR + GV_RED_DN + (staged ? tile_bytes(Kmax) : 0);
}

// STAGED: the CTA's whole weight tile (16 code rows, their scales and biases) comes into shared
// memory by bulk copies issued by one thread as soon as the group is known, so every byte of
// the tile is in flight at once and no registers hold loads in flight (more CTAs per SM); the
// arithmetic and its order are the same as the register-streaming form (!STAGED, used when a
// matrix is not 16-row tiled or not 16-byte aligned).
// Waits for the staged tile; false (recorded in a.err, every copy drained, bounded) when it
// never arrives. Whole CTA.
__device__ __forceinline__ bool gv_tile_wait(uint64_t* bar, int* berr, int* err) {
  const bool ok = __syncthreads_and(mbar_wait(bar, 0, berr, 1, GV_WAIT_CYCLES));
  if (!ok && threadIdx.x == 0) {
    if (err) atomicCAS(err, 0, 0x47);  // 'G': a staged GEMV tile never arrived
    for (const long long t0 = clock64(); !mbar_try_wait(bar, 0) && clock64() - t0 < GV_WAIT_CYCLES;) {
    }
  }
  return ok;
}

// xg[t, g] = the 64-group sum of x row t that the gate/up kernel's fold needs, computed once
// per forward instead of once per 16-row tile (every tile of an expert used to recompute it):
// four lanes per (token, group), each xsum16 over its 16 values, then the same two butterfly
// adds as the gate/up kernel's in-register form, so the sums have the same bits.
__global__ void __launch_bounds__(256) token_group_sums_kernel(const __nv_bfloat16* __restrict__ x,
                                                              int T, int H,
                                                              float* __restrict__ xg) {
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  const int gpr = H / 64;
  const long long pairs = (long long)T * gpr;
  const int c4 = threadIdx.x & 3;
  // every lane of a warp runs the same number of iterations (the shuffles need them all)
  const long long stride = (long long)gridDim.x * (blockDim.x / 4);
  for (long long i0 = (long long)blockIdx.x * (blockDim.x / 4); i0 < pairs; i0 += stride) {
    const long long i = i0 + (threadIdx.x >> 2);
    const bool ok = i < pairs;
    uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
    if (ok) {
      const int t = (int)(i / gpr), gg = (int)(i % gpr);
      const __nv_bfloat16* xr = x + (size_t)t * H + gg * 64 + 16 * c4;
      xa0 = *reinterpret_cast<const uint4*>(xr);
      xa1 = *reinterpret_cast<const uint4*>(xr + 8);
    }
    float xs = xsum16(xa0, xa1);
    xs += __shfl_xor_sync(0xffffffffu, xs, 1);
    xs += __shfl_xor_sync(0xffffffffu, xs, 2);
    if (ok && c4 == 0) xg[i] = xs;
  }
}

template <bool STAGED>
__global__ void __launch_bounds__(GV_WARPS * 32) moe_gemv_gateup_kernel(GemvArgs a) {
  extern __shared__ __align__(128) uint8_t gv_smem[];
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  float (*red)[2][32][4] = reinterpret_cast<float (*)[2][32][4]>(gv_smem + GV_HDR);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int na = a.active[0];
  if ((int)blockIdx.y >= na) return;
  const int g = a.active[1 + blockIdx.y];
  const bool sh = (g == a.E);
  const int Ig = sh ? a.I_sh : a.I;
  const int m0 = blockIdx.x * 16;
  if (m0 >= Ig) return;
  const int H = a.H;
  const int wpr = H / 8;         // words per weight row
  const int gpr = H / 64;        // groups per row
  const uint32_t* gq = sh ? a.sg_q : a.g_q + (size_t)g * a.I * wpr;
  const uint32_t* uq = sh ? a.su_q : a.u_q + (size_t)g * a.I * wpr;
  const __nv_bfloat16* gs = sh ? a.sg_s : a.g_s + (size_t)g * a.I * gpr;
  const __nv_bfloat16* gb = sh ? a.sg_b : a.g_b + (size_t)g * a.I * gpr;
  const __nv_bfloat16* us = sh ? a.su_s : a.u_s + (size_t)g * a.I * gpr;
  const __nv_bfloat16* ub = sh ? a.su_b : a.u_b + (size_t)g * a.I * gpr;
  const int r = lane >> 2, c4 = lane & 3;
  const int ra = m0 + r, rb = m0 + r + 8;
  // staged: rows r / r + 8 of the two tiles, and their scale and bias rows, in shared memory
  uint8_t* ring = gv_smem + GV_HDR + GV_RED_GU;
  const uint32_t tb = tile_bytes(H), pitch = tile_pitch(H);
  if constexpr (STAGED) {
    uint64_t* bar = reinterpret_cast<uint64_t*>(gv_smem);
    int* berr = reinterpret_cast<int*>(gv_smem + 8);
    if (threadIdx.x == 0) {
      *berr = 0;
      mbar_init(bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(bar, 2u * tile_bulk_bytes(H));
      tile_load_bulk(ring, gq, gs, gb, m0, H, bar);
      tile_load_bulk(ring + tb, uq, us, ub, m0, H, bar);
    }
    __syncthreads();  // the barrier is initialised before anyone polls it
    if (!gv_tile_wait(bar, berr, a.err)) return;
  }
  const __nv_bfloat16* tgs = reinterpret_cast<const __nv_bfloat16*>(ring + tile_sc_off(H));
  const __nv_bfloat16* tus = reinterpret_cast<const __nv_bfloat16*>(ring + tb + tile_sc_off(H));
  const int row0 = a.offsets[g], cnt = a.offsets[g + 1] - row0;
  for (int t8 = 0; t8 < cnt; t8 += 8) {
    const int tn = t8 + r;  // this thread's B-fragment token (row of the group)
    const bool tval = tn < cnt;
    const int tok = tval ? row_token(a.perm[row0 + tn], a.P, a.k) : 0;
    const __nv_bfloat16* xrow = a.x + (size_t)tok * H;
    // the group sums of the C-layout columns 2c4, 2c4 + 1 (rows 2c4, 2c4 + 1 of this tile)
    const int tc0 = __shfl_sync(0xffffffffu, tval ? tok : -1, (2 * c4) * 4);
    const int tc1 = __shfl_sync(0xffffffffu, tval ? tok : -1, (2 * c4 + 1) * 4);
    const float* xg0 = tc0 >= 0 ? a.xg + (size_t)tc0 * gpr : nullptr;
    const float* xg1 = tc1 >= 0 ? a.xg + (size_t)tc1 * gpr : nullptr;
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll(STAGED ? 1 : 2)
    for (int gg = warp; gg < gpr; gg += GV_WARPS) {
      const size_t wo = (size_t)gg * 8 + 2 * c4;
      uint2 g0, g8, u0, u8;
      if constexpr (STAGED) {
        const uint32_t o0 = r * pitch + gg * 32 + c4 * 8, o8 = o0 + 8 * pitch;
        g0 = *reinterpret_cast<const uint2*>(ring + o0);
        g8 = *reinterpret_cast<const uint2*>(ring + o8);
        u0 = *reinterpret_cast<const uint2*>(ring + tb + o0);
        u8 = *reinterpret_cast<const uint2*>(ring + tb + o8);
      } else {
        g0 = *reinterpret_cast<const uint2*>(gq + (size_t)ra * wpr + wo);
        g8 = *reinterpret_cast<const uint2*>(gq + (size_t)rb * wpr + wo);
        u0 = *reinterpret_cast<const uint2*>(uq + (size_t)ra * wpr + wo);
        u8 = *reinterpret_cast<const uint2*>(uq + (size_t)rb * wpr + wo);
      }
      uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
      if (tval) {
        xa0 = *reinterpret_cast<const uint4*>(xrow + gg * 64 + 16 * c4);
        xa1 = *reinterpret_cast<const uint4*>(xrow + gg * 64 + 16 * c4 + 8);
      }
      // the columns' group sums (token_group_sums_kernel; 0 past the group's rows)
      const float xs0 = xg0 ? xg0[gg] : 0.f;
      const float xs1 = xg1 ? xg1[gg] : 0.f;
      float sg0, sg8, bg0, bg8, su0, su8, bu0, bu8;
      if constexpr (STAGED) {  // the tile's scales [16][gpr], then its biases [16][gpr]
        const int i0 = r * gpr + gg, i8 = i0 + 8 * gpr, nb = 16 * gpr;
        sg0 = bf2f(tgs[i0]); sg8 = bf2f(tgs[i8]); bg0 = bf2f(tgs[nb + i0]); bg8 = bf2f(tgs[nb + i8]);
        su0 = bf2f(tus[i0]); su8 = bf2f(tus[i8]); bu0 = bf2f(tus[nb + i0]); bu8 = bf2f(tus[nb + i8]);
      } else {
        sg0 = bf2f(gs[(size_t)ra * gpr + gg]); sg8 = bf2f(gs[(size_t)rb * gpr + gg]);
        bg0 = bf2f(gb[(size_t)ra * gpr + gg]); bg8 = bf2f(gb[(size_t)rb * gpr + gg]);
        su0 = bf2f(us[(size_t)ra * gpr + gg]); su8 = bf2f(us[(size_t)rb * gpr + gg]);
        bu0 = bf2f(ub[(size_t)ra * gpr + gg]); bu8 = bf2f(ub[(size_t)rb * gpr + gg]);
      }
      float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
      group_mma(dg, g0, g8, xa0, xa1);
      group_mma(du, u0, u8, xa0, xa1);
      accg[0] += sg0 * dg[0] + bg0 * xs0;
      accg[1] += sg0 * dg[1] + bg0 * xs1;
      accg[2] += sg8 * dg[2] + bg8 * xs0;
      accg[3] += sg8 * dg[3] + bg8 * xs1;
      accu[0] += su0 * du[0] + bu0 * xs0;
      accu[1] += su0 * du[1] + bu0 * xs1;
      accu[2] += su8 * du[2] + bu8 * xs0;
      accu[3] += su8 * du[3] + bu8 * xs1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      red[warp][0][lane][j] = accg[j];
      red[warp][1][lane][j] = accu[j];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float gv = 0.f, uv = 0.f;
#pragma unroll
        for (int w = 0; w < GV_WARPS; ++w) {
          gv += red[w][0][lane][j];
          uv += red[w][1][lane][j];
        }
        const int col = t8 + 2 * c4 + (j & 1);   // group row (token tile column)
        const int n = (j < 2) ? ra : rb;        // intermediate index
        if (col < cnt) {
          const float gr = round_bf16(gv), ur = round_bf16(uv);
          const float sig = round_bf16(1.0f / (1.0f + expf(-gr)));
          const float sl = round_bf16(gr * sig);
          a.h[(size_t)(row0 + col) * a.h_stride + n] = __float2bfloat16_rn(sl * ur);
        }
      }
    }
    __syncthreads();
  }
}

template <bool STAGED>
__global__ void __launch_bounds__(GV_WARPS * 32) moe_gemv_down_kernel(GemvArgs a) {
  extern __shared__ __align__(128) uint8_t gv_smem[];
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  float (*red)[32][4] = reinterpret_cast<float (*)[32][4]>(gv_smem + GV_HDR);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int na = a.active[0];
  if ((int)blockIdx.y >= na) return;
  const int g = a.active[1 + blockIdx.y];
  const bool sh = (g == a.E);
  const int Kg = sh ? a.I_sh : a.I;  // reduction length
  const int H = a.H;
  const int m0 = blockIdx.x * 16;
  if (m0 >= H) return;
  const int row0 = a.offsets[g], cnt = a.offsets[g + 1] - row0;
  const int wpr = Kg / 8, gpr = Kg / 64;
  const uint32_t* dq = sh ? a.sd_q : a.d_q + (size_t)g * H * (a.I / 8);
  const __nv_bfloat16* ds = sh ? a.sd_s : a.d_s + (size_t)g * H * (a.I / 64);
  const __nv_bfloat16* db = sh ? a.sd_b : a.d_b + (size_t)g * H * (a.I / 64);
  const int r = lane >> 2, c4 = lane & 3;
  const int ra = m0 + r, rb = m0 + r + 8;
  uint8_t* tile = gv_smem + GV_HDR + GV_RED_DN;
  const uint32_t pitch = tile_pitch(Kg);
  if constexpr (STAGED) {
    uint64_t* bar = reinterpret_cast<uint64_t*>(gv_smem);
    int* berr = reinterpret_cast<int*>(gv_smem + 8);
    if (threadIdx.x == 0) {
      *berr = 0;
      mbar_init(bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(bar, tile_bulk_bytes(Kg));
      tile_load_bulk(tile, dq, ds, db, m0, Kg, bar);
    }
    __syncthreads();  // the barrier is initialised before anyone polls it
    if (!gv_tile_wait(bar, berr, a.err)) return;
  }
  const __nv_bfloat16* tds = reinterpret_cast<const __nv_bfloat16*>(tile + tile_sc_off(Kg));

  for (int t8 = 0; t8 < cnt; t8 += 8) {
    const int tn = t8 + r;
    const bool tval = tn < cnt;
    const __nv_bfloat16* hrow = a.h + (size_t)(row0 + (tval ? tn : 0)) * a.h_stride;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll(STAGED ? 1 : 2)
    for (int gg = warp; gg < gpr; gg += GV_WARPS) {
      const size_t wo = (size_t)gg * 8 + 2 * c4;
      uint2 w0, w8;
      if constexpr (STAGED) {
        const uint32_t o0 = r * pitch + gg * 32 + c4 * 8;
        w0 = *reinterpret_cast<const uint2*>(tile + o0);
        w8 = *reinterpret_cast<const uint2*>(tile + o0 + 8 * pitch);
      } else {
        w0 = *reinterpret_cast<const uint2*>(dq + (size_t)ra * wpr + wo);
        w8 = *reinterpret_cast<const uint2*>(dq + (size_t)rb * wpr + wo);
      }
      uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
      if (tval) {
        xa0 = *reinterpret_cast<const uint4*>(hrow + gg * 64 + 16 * c4);
        xa1 = *reinterpret_cast<const uint4*>(hrow + gg * 64 + 16 * c4 + 8);
      }
      float xs = xsum16(xa0, xa1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 2);
      const float xs0 = __shfl_sync(0xffffffffu, xs, (2 * c4) * 4);
      const float xs1 = __shfl_sync(0xffffffffu, xs, (2 * c4 + 1) * 4);
      float s0, s8, b0, b8;
      if constexpr (STAGED) {
        const int i0 = r * gpr + gg, i8 = i0 + 8 * gpr, nb = 16 * gpr;
        s0 = bf2f(tds[i0]); s8 = bf2f(tds[i8]); b0 = bf2f(tds[nb + i0]); b8 = bf2f(tds[nb + i8]);
      } else {
        s0 = bf2f(ds[(size_t)ra * gpr + gg]); s8 = bf2f(ds[(size_t)rb * gpr + gg]);
        b0 = bf2f(db[(size_t)ra * gpr + gg]); b8 = bf2f(db[(size_t)rb * gpr + gg]);
      }
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      group_mma(d, w0, w8, xa0, xa1);
      acc[0] += s0 * d[0] + b0 * xs0;
      acc[1] += s0 * d[1] + b0 * xs1;
      acc[2] += s8 * d[2] + b8 * xs0;
      acc[3] += s8 * d[3] + b8 * xs1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[warp][lane][j] = acc[j];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < GV_WARPS; ++w) v += red[w][lane][j];
        const int col = t8 + 2 * c4 + (j & 1);
        const int n = (j < 2) ? ra : rb;
        if (col < cnt) {
          const int p = a.perm[row0 + col];
          // gather_qmm's bf16 output per pick row (shared rows follow the routed ones), or
          // (expert parallel) weighted into the source rank's combine row
          if (a.ep.on) {
            float wt;
            __nv_bfloat16* orow = ep_ret_row(a.ep, p, a.k, H, &wt);
            orow[n] = __float2bfloat16_rn(round_bf16(v) * wt);
          } else {
            a.ypick[(size_t)p * H + n] = __float2bfloat16_rn(v);
          }
        }
      }
    }
    __syncthreads();
  }
  if (a.ep.on) __threadfence_system();  // peer stores visible before the signal
}

// The staged kernels need whole 16-row tiles and 16-byte aligned rows, scale and bias blocks
// (every tile's rows start at a multiple of 16 rows); otherwise the register-streaming form.
static bool gv_aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool gv_stageable(const GemvArgs& a) {
  bool ok = a.H % 16 == 0 && a.I % 16 == 0 && a.I_sh % 16 == 0;
  const void* ps[] = {a.g_q, a.u_q, a.d_q, a.g_s, a.g_b, a.u_s, a.u_b, a.d_s, a.d_b,
                      a.sg_q, a.su_q, a.sd_q, a.sg_s, a.sg_b, a.su_s, a.su_b, a.sd_s, a.sd_b};
  for (const void* p : ps) ok = ok && (p == nullptr || gv_aligned(p));
  return ok;
}

template <typename K>
static cudaError_t gv_launch(K kernel, dim3 grid, uint32_t smem, cudaStream_t s, const GemvArgs& a) {
  if (smem > 48u * 1024u) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(kernel, grid, dim3(GV_WARPS * 32), smem, s, a);
}

int launch_gemv(const GemvArgs& a, int max_groups, cudaStream_t s) {
  if (max_groups <= 0) return LG_OK;
  const bool staged = gv_stageable(a);
  const int Imax = a.I > a.I_sh ? a.I : a.I_sh;
  dim3 g1((Imax + 15) / 16, max_groups);
  if (a.T > 0) {
    const long long pairs = (long long)a.T * (a.H / 64);
    long long blocks = (pairs + 63) / 64;  // 64 (token, group) pairs per 256-thread block
    if (blocks > 8LL * device_sm_count()) blocks = 8LL * device_sm_count();
    LG_CUDA_TRY(launch_k(token_group_sums_kernel, dim3((unsigned)blocks), dim3(256), 0, s, a.x,
                         a.T, a.H, a.xg));
    LG_LAUNCH_CHECK("token_group_sums");
  }
  prof_begin("experts_gateup", s);
  LG_CUDA_TRY(staged ? gv_launch(moe_gemv_gateup_kernel<true>, g1, gv_smem_gu(a.H, true), s, a)
                     : gv_launch(moe_gemv_gateup_kernel<false>, g1, gv_smem_gu(a.H, false), s, a));
  prof_end("experts_gateup", s);
  LG_LAUNCH_CHECK("moe_gemv_gateup");
  dim3 g2((a.H + 15) / 16, max_groups);
  prof_begin("experts_down", s);
  LG_CUDA_TRY(staged ? gv_launch(moe_gemv_down_kernel<true>, g2, gv_smem_dn(Imax, true), s, a)
                     : gv_launch(moe_gemv_down_kernel<false>, g2, gv_smem_dn(Imax, false), s, a));
  prof_end("experts_down", s);
  LG_LAUNCH_CHECK("moe_gemv_down");
  return LG_OK;
}

}  // namespace lg
