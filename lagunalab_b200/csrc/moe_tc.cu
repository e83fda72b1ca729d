// Prefill-size MoE expert products on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Dispatch: the picks, ordered by expert (routing plan), are gathered into an
// expert-contiguous activation matrix (the token-to-expert dispatch, laguna.py:149 via
// SwitchGLU's sorted path); the shared expert's T rows follow the routed ones.
//
// Grouped GEMM (one persistent CTA per SM, tiles of 128 rows x 256 columns x K, K-step 64 =
// one quantization group):
//   warp 0      TMA: activation tile (128 x 64 bf16, 128-byte swizzle) into a 3-stage ring
//   warp 2      TMA: packed 4-bit weight rows (256 rows x 32 bytes) into a staging ring
//   warps 4-11  dequantize the staged words in registers (one B row per thread),
//               value = scale * code + bias in bf16
//               (one LOP3 + SUB + FMA per two values), and store the bf16 B tile in the
//               128-byte-swizzled K-major layout the tensor core reads
//   warp 1      one thread issues tcgen05.mma (M 128, N 256, K 16, bf16 -> fp32) into one of
//               two TMEM accumulators (2 x 256 columns) and commits stage / tile barriers
//   warps 12-15 epilogue: tcgen05.ld of the accumulator; gate/up: SwiGLU with the MLX bf16
//               rounding points (laguna.py:122) -> h; down: y -> bf16 stored per pick row
//               (routed picks, then the shared expert's rows); the weighted combine
//               (laguna.py:149-150) is a separate fixed-order pass over those rows
// The two TMEM accumulators let the epilogue of one tile overlap the MMAs of the next.
//
// K order: inside every aligned 8-wide K chunk the operands are stored in the order
// (0,4,1,5,2,6,3,7), the order in which one LOP3 splits a 32-bit MLX word into bf16 pairs.
// The dispatch gather writes activations in that order and the gate/up epilogue writes h in
// it, so the dequantizer never shuffles nibbles. K is contracted, so results are unchanged.
//
// Every mbarrier wait is bounded (tc::mbar_wait): on expiry the kernel records an error code
// in the workspace status word and all roles leave their loops.
#include <cudaTypedefs.h>

#include "moe.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace lg {

using namespace tc;

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64;
constexpr int TC_NA = 3;  // activation (A) stages
constexpr int TC_NS = 3;  // dequantized weight (B) stages
constexpr int TC_NP = 4;  // packed-weight stages
constexpr int TC_THREADS = 512;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;  // 32 KB
constexpr int TC_P_BYTES = TC_BN * TC_BK / 2;  // 8 KB
constexpr int TC_NBAR = 2 * TC_NA + 2 * TC_NS + 2 * TC_NP + 5;
// down-epilogue staging: per epilogue warp 32 rows x 64 bf16 columns, rows 144 bytes apart
constexpr int TC_OUT_PITCH = 144;
constexpr int TC_OUT_BYTES = 4 * 32 * TC_OUT_PITCH;
constexpr size_t TC_SMEM = 1024 + TC_NA * TC_A_BYTES + TC_NS * TC_B_BYTES + TC_NP * TC_P_BYTES +
                           TC_NBAR * 8 + 16 + 16 + TC_OUT_BYTES;

#ifdef LG_TC_PROFILE
// Diagnostic build only: cycles each role spends waiting, per CTA (16 counters).
__device__ long long* g_tc_stats = nullptr;
#define TC_T0() const long long tc_t0_ = clock64()
#define TC_ACC(slot) \
  do { if (g_tc_stats) atomicAdd((unsigned long long*)&g_tc_stats[(GATEUP ? 0 : 4096) + blockIdx.x * 16 + (slot)], \
                                 (unsigned long long)(clock64() - tc_t0_)); } while (0)
#else
#define TC_T0() ((void)0)
#define TC_ACC(slot) ((void)0)
#endif

struct TcArgs {
  const int4* tiles;  // {group, m0, n-tile, 0}
  const int* ntiles;
  const int32_t* offsets;
  const int32_t* perm;
  int E, P, k, H, I, I_sh;
  // scales / biases: matrix 0 (gate or down) and matrix 1 (up), routed and shared
  const __nv_bfloat16 *s0, *b0, *s1, *b1, *ss0, *sb0, *ss1, *sb1;
  __nv_bfloat16* h;
  int h_stride;
  __nv_bfloat16* ypick;  // [rows, H] per-pick down outputs (pick id order)
  EpRet ep;              // expert-parallel return of the down outputs (replaces ypick)
  int* err;
};

__device__ __forceinline__ uint32_t nib2(uint32_t w, int shift) {
  uint32_t r, v = w >> shift;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;
}

// bf16x2 (128 + c) -> scale * c + bias, rounded once (FMA) after an exact subtract.
__device__ __forceinline__ uint32_t deq2(uint32_t v, uint32_t s2, uint32_t b2) {
  uint32_t c, r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(v), "r"(0x43004300u));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(c), "r"(s2), "r"(b2));
  return r;
}

__device__ __forceinline__ uint4 deq_word(uint32_t w, uint32_t s2, uint32_t b2) {
  return make_uint4(deq2(nib2(w, 0), s2, b2), deq2(nib2(w, 4), s2, b2), deq2(nib2(w, 8), s2, b2),
                    deq2(nib2(w, 12), s2, b2));
}

__device__ __forceinline__ uint32_t bf2_splat(__nv_bfloat16 v) {
  uint16_t u = *reinterpret_cast<uint16_t*>(&v);
  return (uint32_t)u | ((uint32_t)u << 16);
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float swiglu_mlx(float g, float u) {
  const float gr = round_bf16(g), ur = round_bf16(u);
  const float sig = round_bf16(1.0f / (1.0f + expf(-gr)));
  return round_bf16(gr * sig) * ur;
}

template <bool GATEUP>
__global__ void __launch_bounds__(TC_THREADS, 1)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w0,
                  const __grid_constant__ CUtensorMap tm_w1,
                  const __grid_constant__ CUtensorMap tm_sw0,
                  const __grid_constant__ CUtensorMap tm_sw1, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = sA + TC_NA * TC_A_BYTES;
  uint32_t* sP = reinterpret_cast<uint32_t*>(sB + TC_NS * TC_B_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sP) + TC_NP * TC_P_BYTES);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + TC_NA;
  uint64_t* b_full = a_empty + TC_NA;
  uint64_t* s_empty = b_full + TC_NS;  // B stage free
  uint64_t* p_full = s_empty + TC_NS;
  uint64_t* p_empty = p_full + TC_NP;
  uint64_t* t_full = p_empty + TC_NP;
  uint64_t* t_empty = t_full + 2;
  uint64_t* teardown = t_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  uint8_t* sOut = reinterpret_cast<uint8_t*>(  // 16-byte aligned, within the 32 bytes reserved
      (reinterpret_cast<uintptr_t>(tmem_slot) + 4 + 15) & ~static_cast<uintptr_t>(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = a.err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_NA; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < TC_NS; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&s_empty[i], 1);
    }
    for (int i = 0; i < TC_NP; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 1);
    }
    mbar_init(teardown, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = *a.ntiles;
  const int H = a.H;

  auto ksteps = [&](int g) -> int { return GATEUP ? H / TC_BK : ((g == a.E) ? a.I_sh : a.I) / TC_BK; };

  if (warp == 0) {
    // ---------------- activation TMA producer ----------------
    if (lane == 0) prefetch_tmap(&tm_a);
    int step = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int4 tl = a.tiles[t];
      const int row = a.offsets[tl.x] + tl.y;
      const int ks = ksteps(tl.x);
      for (int kb = 0; kb < ks && ok; ++kb, ++step) {
        const int s = step % TC_NA;
        const uint32_t ph = (step / TC_NA) & 1;
        if (lane == 0) {
          TC_T0();
          ok = mbar_wait(&a_empty[s], ph ^ 1, err, 1);
          TC_ACC(6);
          if (ok) {
            mbar_arrive_expect_tx(&a_full[s], TC_A_BYTES);
            tma_load_2d(sA + s * TC_A_BYTES, &tm_a, &a_full[s], kb * TC_BK, row);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    }
  } else if (warp == 2) {
    // ---------------- packed-weight TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_w0);
      prefetch_tmap(&tm_w1);
      prefetch_tmap(&tm_sw0);
      prefetch_tmap(&tm_sw1);
    }
    int step = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int4 tl = a.tiles[t];
      const int g = tl.x, nt = tl.z;
      const bool sh = (g == a.E);
      const int ks = ksteps(g);
      const CUtensorMap* m0 = sh ? &tm_sw0 : &tm_w0;
      const CUtensorMap* m1 = GATEUP ? (sh ? &tm_sw1 : &tm_w1) : m0;
      int r0, r1;
      if (GATEUP) {
        r0 = (sh ? 0 : g * a.I) + nt * 128;
        r1 = r0;
      } else {
        r0 = (sh ? 0 : g * H) + nt * 256;
        r1 = r0 + 128;
      }
      for (int kb = 0; kb < ks && ok; ++kb, ++step) {
        const int p = step % TC_NP;
        const uint32_t ph = (step / TC_NP) & 1;
        if (lane == 0) {
          TC_T0();
          ok = mbar_wait(&p_empty[p], ph ^ 1, err, 2);
          TC_ACC(7);
          if (ok) {
            mbar_arrive_expect_tx(&p_full[p], TC_P_BYTES);
            uint32_t* dst = sP + p * (TC_P_BYTES / 4);
            tma_load_2d(dst, m0, &p_full[p], kb * 8, r0);
            tma_load_2d(dst + 128 * 8, m1, &p_full[p], kb * 8, r1);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_bf16(TC_BM, TC_BN);
    int step = 0, it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
      const int4 tl = a.tiles[t];
      const int ks = ksteps(tl.x);
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (lane == 0) {
        TC_T0();
        ok = mbar_wait(&t_empty[acc], aph ^ 1, err, 3);
        TC_ACC(2);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * TC_BN;
      for (int kb = 0; kb < ks && ok; ++kb, ++step) {
        const int sa = step % TC_NA, s = step % TC_NS;
        const uint32_t pha = (step / TC_NA) & 1, ph = (step / TC_NS) & 1;
        if (lane == 0) {
          {
            TC_T0();
            ok = mbar_wait(&a_full[sa], pha, err, 4);
            TC_ACC(0);
          }
          if (ok) {
            TC_T0();
            ok = mbar_wait(&b_full[s], ph, err, 5);
            TC_ACC(1);
          }
          if (ok) {
            tc_fence_after();
            const uint64_t ad = sw128_desc(smem_u32(sA + sa * TC_A_BYTES));
            const uint64_t bd = sw128_desc(smem_u32(sB + s * TC_B_BYTES));
#pragma unroll
            for (int k = 0; k < TC_BK / 16; ++k)
              umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
            umma_commit(&a_empty[sa]);
            umma_commit(&s_empty[s]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();
      }
      if (lane == 0 && ok) umma_commit(&t_full[acc]);
      __syncwarp();
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------- dequantizer: one B row per thread (256 rows) ----------------
    const int dt = threadIdx.x - 128;  // B-tile row
    int step = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int4 tl = a.tiles[t];
      const int g = tl.x, nt = tl.z;
      const bool sh = (g == a.E);
      const int ks = ksteps(g);
      const int gpr = ks;  // groups per weight row = K / 64
      const __nv_bfloat16 *sc, *bi;
      if (GATEUP) {  // rows 0-127: gate rows, 128-255: up rows, of n-tile rows nt*128 + (dt % 128)
        const size_t base = sh ? 0 : (size_t)g * a.I * gpr;
        const size_t row = (size_t)(nt * 128 + (dt & 127)) * gpr;
        const bool up = dt >= 128;
        sc = (up ? (sh ? a.ss1 : a.s1 + base) : (sh ? a.ss0 : a.s0 + base)) + row;
        bi = (up ? (sh ? a.sb1 : a.b1 + base) : (sh ? a.sb0 : a.b0 + base)) + row;
      } else {  // down rows nt*256 + dt
        const size_t base = sh ? 0 : (size_t)g * H * gpr;
        const size_t row = (size_t)(nt * 256 + dt) * gpr;
        sc = (sh ? a.ss0 : a.s0 + base) + row;
        bi = (sh ? a.sb0 : a.b0 + base) + row;
      }
      __nv_bfloat16 ns = sc[0], nb = bi[0];
      for (int kb = 0; kb < ks && ok; ++kb, ++step) {
        const uint32_t s2 = bf2_splat(ns), b2 = bf2_splat(nb);
        if (kb + 1 < ks) {  // next group's scale/bias, issued before the waits
          ns = sc[kb + 1];
          nb = bi[kb + 1];
        }
        const int p = step % TC_NP, s = step % TC_NS;
        const uint32_t pph = (step / TC_NP) & 1, sph = (step / TC_NS) & 1;
        // wait for the packed words and for the operand stage, then load, dequantize and
        // store; the staging stage is released only after the stores, which depend on the
        // loaded words, so no later TMA into it can race with these loads
        bool got;
        {
          TC_T0();
          got = mbar_wait(&p_full[p], pph, err, 6);
          if (dt == 0) TC_ACC(3);
        }
        if (got) {
          TC_T0();
          got = mbar_wait(&s_empty[s], sph ^ 1, err, 7);
          if (dt == 0) TC_ACC(4);
        }
        if (got) {
          // staged rows are 32 bytes, written by TMA with the 32-byte swizzle: the 16-byte half
          // c of row r sits at half c ^ ((r >> 2) & 1)
          const uint32_t* src = sP + p * (TC_P_BYTES / 4) + dt * 8;
          const int x0 = ((dt >> 2) & 1) * 4;
          const uint4 wa = *reinterpret_cast<const uint4*>(src + x0);
          const uint4 wb = *reinterpret_cast<const uint4*>(src + (4 - x0));
          uint8_t* dst = sB + s * TC_B_BYTES + dt * 128;
          const uint32_t wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(dst + ((j ^ (dt & 7)) << 4)) = deq_word(wv[j], s2, b2);
          // order this thread's generic-proxy stores before the tensor core's async-proxy reads
          fence_proxy_async_smem();
        }
        // all 256 threads have stored and fenced: one thread releases the staging stage and
        // publishes the operand stage
        {
          TC_T0();
          ok = bar_and_n<1, 256>(got);
          if (dt == 0) TC_ACC(5);
        }
        if (!ok) break;
        if (dt == 0) mbar_arrive(&p_empty[p]);
        if (dt == 0) mbar_arrive(&b_full[s]);
      }
    }
  } else if (warp >= 12) {
    // ---------------- epilogue (warps 12-15: TMEM lane quarters 0-3) ----------------
    const int q = warp & 3;
    const int er = 32 * q + lane;  // tile row = TMEM lane
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
      const int4 tl = a.tiles[t];
      const int g = tl.x, m0 = tl.y, nt = tl.z;
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      {
        TC_T0();
        ok = bar_and_n<2, 128>(mbar_wait(&t_full[acc], aph, err, 8));
        if (er == 0) TC_ACC(8);
      }
      if (!ok) break;  // uniform over the epilogue warps: tcgen05.ld is a warp-collective
      tc_fence_after();
      const int row0 = a.offsets[g], cnt = a.offsets[g + 1] - row0;
      const int gm = m0 + er;
      const bool valid = gm < cnt;
      const int R = row0 + gm;
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + acc * TC_BN;
      if (GATEUP) {
        __nv_bfloat16* hrow = a.h + (size_t)R * a.h_stride + nt * 128;
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t gv[16], uv[16];
          tmem_ld16(taddr + c, gv);
          tmem_ld16(taddr + 128 + c, uv);
          tmem_ld_wait(gv, uv);
          if (valid) {
            float hv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) hv[j] = swiglu_mlx(__uint_as_float(gv[j]), __uint_as_float(uv[j]));
            // store in the (0,4,1,5,2,6,3,7) chunk order read by the down product
            uint4 o0 = make_uint4(pack_bf2(hv[0], hv[4]), pack_bf2(hv[1], hv[5]),
                                  pack_bf2(hv[2], hv[6]), pack_bf2(hv[3], hv[7]));
            uint4 o1 = make_uint4(pack_bf2(hv[8], hv[12]), pack_bf2(hv[9], hv[13]),
                                  pack_bf2(hv[10], hv[14]), pack_bf2(hv[11], hv[15]));
            *reinterpret_cast<uint4*>(hrow + c) = o0;
            *reinterpret_cast<uint4*>(hrow + c + 8) = o1;
          }
        }
      } else {
        // down: gather_qmm's bf16 output per pick row (shared rows after the routed ones), or
        // (expert parallel) bf16(bf16(y) * w) into the source rank's combine row. 64 columns
        // at a time go through this warp's shared-memory rows, so that each store instruction
        // writes whole 128-byte lines (8 lanes per row, 4 rows per instruction) — also to a
        // peer GPU's memory over NVLink
        const int n0 = nt * 256;
        __nv_bfloat16* orow = nullptr;
        float wt = 1.0f;
        if (valid) {
          const int p = a.perm[R];
          orow = a.ep.on ? ep_ret_row(a.ep, p, a.k, H, &wt) : a.ypick + (size_t)p * H;
        }
        uint8_t* stg = sOut + q * (32 * TC_OUT_PITCH);
        uint8_t* mine = stg + lane * TC_OUT_PITCH;
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 64) {
#pragma unroll 1
          for (int cc = 0; cc < 64; cc += 16) {
            uint32_t yv[16];
            tmem_ld16(taddr + c0 + cc, yv);
            tmem_ld_wait(yv);
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = __uint_as_float(yv[j]);
            if (a.ep.on) {
#pragma unroll
              for (int j = 0; j < 16; ++j) y[j] = round_bf16(y[j]) * wt;
            }
            uint4* s4 = reinterpret_cast<uint4*>(mine + cc * 2);
            s4[0] = make_uint4(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]), pack_bf2(y[4], y[5]),
                               pack_bf2(y[6], y[7]));
            s4[1] = make_uint4(pack_bf2(y[8], y[9]), pack_bf2(y[10], y[11]),
                               pack_bf2(y[12], y[13]), pack_bf2(y[14], y[15]));
          }
          __syncwarp();
#pragma unroll
          for (int w8 = 0; w8 < 8; ++w8) {
            const int rr = w8 * 4 + (lane >> 3), seg = lane & 7;
            const unsigned long long dst =
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow), rr);
            if (dst) {
              const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * TC_OUT_PITCH + seg * 16);
              *reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst) + (size_t)(n0 + c0) * 2 +
                                        seg * 16) = v;
            }
          }
          __syncwarp();
        }
      }
      // every epilogue thread has waited for its TMEM loads; one arrive hands the accumulator
      // back to the MMA issuer after all 128 have passed the barrier
      tc_fence_before();
      bar_and_n<2, 128>(true);
      if (er == 0) mbar_arrive(&t_empty[acc]);
    }
  }

  // ---------------- teardown: every MMA retired before TMEM is released ----------------
  if (!GATEUP && a.ep.on) __threadfence_system();  // peer stores visible before the signal
  __syncthreads();
#ifdef LG_TC_PROFILE
  if (threadIdx.x == 0 && g_tc_stats) g_tc_stats[(GATEUP ? 0 : 4096) + blockIdx.x * 16 + 9] = clock64();
#endif
  if (warp == 1) {
    if (lane == 0) {
      umma_commit(teardown);
      mbar_wait(teardown, 0, err, 9);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// Dispatch gather: row R of the expert-contiguous activation matrix = x[token(perm[R])] with
// every 8-element chunk stored in (0,4,1,5,2,6,3,7) order. One warp per row.
__global__ void __launch_bounds__(256) dispatch_gather_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const int32_t* __restrict__ perm,
                                                              const int32_t* __restrict__ offsets,
                                                              int G, int P, int k, int H,
                                                              int rows_max,
                                                              __nv_bfloat16* __restrict__ xp) {
  const int R = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (R >= rows_max || R >= offsets[G]) return;
  const int p = perm[R];
  const int tok = p < P ? p / k : p - P;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok * H);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)R * H);
  for (int c = lane; c < H / 8; c += 32) {
    const uint4 v = src[c];
    uint4 o;
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(o.x) : "r"(v.x), "r"(v.z));
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(o.y) : "r"(v.x), "r"(v.z));
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(o.z) : "r"(v.y), "r"(v.w));
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(o.w) : "r"(v.y), "r"(v.w));
    dst[c] = o;
  }
}

// Tile lists for both products, ordered by group, then n-tile, then m-tile (a group's tiles
// run side by side, so its weights and activations stay in L2). Per-group tile counts are
// scanned across the block, then every thread writes tiles, finding each tile's group by a
// binary search over the scanned counts.
__global__ void __launch_bounds__(512) tc_schedule_kernel(const int32_t* __restrict__ offsets,
                                                          int G, int E, int I, int I_sh, int H,
                                                          int4* __restrict__ tiles_gu,
                                                          int4* __restrict__ tiles_dn,
                                                          int* __restrict__ counts) {
  __shared__ int pre_gu[513], pre_dn[513], mts[512];
  __shared__ int warp_tot[32], tot_gu, tot_dn;
  const int g = threadIdx.x;
  int ngu = 0, ndn = 0, mt = 0;
  if (g < G) {
    const int cnt = offsets[g + 1] - offsets[g];
    mt = (cnt + TC_BM - 1) / TC_BM;
    const int Ig = (g == E) ? I_sh : I;
    ngu = mt * (Ig / 128);
    ndn = mt * (H / 256);
  }
  mts[g] = mt;
  pre_gu[g] = block_excl_scan(ngu, warp_tot, &tot_gu);
  pre_dn[g] = block_excl_scan(ndn, warp_tot, &tot_dn);
  __syncthreads();
  const int ngu_all = tot_gu, ndn_all = tot_dn;
  if (g == 0) {
    counts[0] = ngu_all;
    counts[1] = ndn_all;
  }
  auto group_of = [&](const int* pre, int i) {
    int lo = 0, hi = G - 1;  // last group with pre[group] <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  };
  for (int i = threadIdx.x; i < ngu_all; i += blockDim.x) {
    int gg = group_of(pre_gu, i);
    while (mts[gg] == 0) --gg;  // skip empty groups sharing the same prefix
    const int local = i - pre_gu[gg];
    tiles_gu[i] = make_int4(gg, (local % mts[gg]) * TC_BM, local / mts[gg], 0);
  }
  for (int i = threadIdx.x; i < ndn_all; i += blockDim.x) {
    int gg = group_of(pre_dn, i);
    while (mts[gg] == 0) --gg;
    const int local = i - pre_dn[gg];
    tiles_dn[i] = make_int4(gg, (local % mts[gg]) * TC_BM, local / mts[gg], 0);
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------

// swz: 128 = 128-byte swizzle (bf16 operand tiles), 32 = 32-byte swizzle (packed weight rows)
static int make_map(CUtensorMap* m, const void* base, bool bf16, uint64_t inner, uint64_t rows,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, int swz) {
  return make_map_2d(m, base, bf16, inner, rows, row_bytes, box_inner, box_rows, swz);
}

struct TcWs {
  __nv_bfloat16* xp;
  int4* tiles_gu;
  int4* tiles_dn;
  int* counts;  // [0] gate/up tiles, [1] down tiles, [2] status word
};

static void tc_limits(int T, int H, int I, int I_sh, int E, int k, size_t* rows, size_t* gu,
                      size_t* dn) {
  const size_t P = (size_t)T * k;
  const size_t G = E + (I_sh > 0 ? 1 : 0);
  *rows = P + (I_sh > 0 ? T : 0);
  const size_t mt = *rows / TC_BM + G;
  const int Imax = I > I_sh ? I : I_sh;
  *gu = mt * (Imax / 128 > 0 ? Imax / 128 : 1);
  *dn = mt * (H / 256 > 0 ? H / 256 : 1);
}

static size_t carve_tc(void* base, int T, int H, int I, int I_sh, int E, int k, TcWs* w) {
  size_t rows, gu, dn;
  tc_limits(T, H, I, I_sh, E, k, &rows, &gu, &dn);
  Carver c(base);
  TcWs t;
  t.xp = c.take<__nv_bfloat16>(rows * H);
  t.tiles_gu = c.take<int4>(gu);
  t.tiles_dn = c.take<int4>(dn);
  t.counts = c.take<int>(4);
  if (w) *w = t;
  return align_up(c.used, 256);
}

size_t tc_workspace_bytes(int T, int H, int I, int I_sh, int E, int k) {
  return carve_tc(nullptr, T, H, I, I_sh, E, k, nullptr);
}

bool tc_supported(int H, int I, int I_sh, int E) {
  return H % 256 == 0 && (E == 0 || I % 128 == 0) && I_sh % 128 == 0;
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int launch_tc(const GemvArgs& a, int max_groups, void* tc_ws, cudaStream_t st) {
  if (!tc_supported(a.H, a.I, a.I_sh, a.E))
    return fail(LG_ERR_UNSUPPORTED,
                "tensor-core path needs hidden %% 256 == 0 and intermediate %% 128 == 0 "
                "(H=%d I=%d I_sh=%d)", a.H, a.I, a.I_sh);
  (void)max_groups;
  static bool attr_set = false;
  if (!attr_set) {
    LG_CUDA_TRY(cudaFuncSetAttribute(moe_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)TC_SMEM));
    LG_CUDA_TRY(cudaFuncSetAttribute(moe_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)TC_SMEM));
    attr_set = true;
  }
  TcWs w;
  carve_tc(tc_ws, a.T, a.H, a.I, a.I_sh, a.E, a.k, &w);
  size_t rows, gu, dn;
  tc_limits(a.T, a.H, a.I, a.I_sh, a.E, a.k, &rows, &gu, &dn);
  const int G = a.E + (a.I_sh > 0 ? 1 : 0);
  const int Imax = a.I > a.I_sh ? a.I : a.I_sh;

  LG_CUDA_TRY(cudaMemsetAsync(w.counts, 0, 4 * sizeof(int), st));
  prof_begin("schedule", st);
  tc_schedule_kernel<<<1, 512, 0, st>>>(a.offsets, G, a.E, a.I, a.I_sh, a.H, w.tiles_gu,
                                        w.tiles_dn, w.counts);
  prof_end("schedule", st);
  LG_LAUNCH_CHECK("tc_schedule");
  prof_begin("dispatch", st);
  dispatch_gather_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a.x, a.perm, a.offsets, G,
                                                                     a.P, a.k, a.H, (int)rows,
                                                                     w.xp);
  prof_end("dispatch", st);
  LG_LAUNCH_CHECK("dispatch_gather");

  // tensor maps (the packed words are viewed as uint32 [rows, K/8])
  CUtensorMap ma, mg, mu, msg, msu, mh, md, msd;
  const int H = a.H;
  int rc;
  if ((rc = make_map(&ma, w.xp, true, H, rows, (uint64_t)H * 2, 64, 128, 128))) return rc;
  if ((rc = make_map(&mh, a.h, true, Imax, rows, (uint64_t)a.h_stride * 2, 64, 128, 128))) return rc;
  const void* dummy = w.xp;  // any valid map for absent matrices (never read)
  if (a.E > 0) {
    if ((rc = make_map(&mg, a.g_q, false, H / 8, (uint64_t)a.E * a.I, H / 2, 8, 128, 32))) return rc;
    if ((rc = make_map(&mu, a.u_q, false, H / 8, (uint64_t)a.E * a.I, H / 2, 8, 128, 32))) return rc;
    if ((rc = make_map(&md, a.d_q, false, a.I / 8, (uint64_t)a.E * H, a.I / 2, 8, 128, 32))) return rc;
  } else {
    if ((rc = make_map(&mg, dummy, false, 8, 128, 32, 8, 128, 32))) return rc;
    mu = md = mg;
  }
  if (a.I_sh > 0) {
    if ((rc = make_map(&msg, a.sg_q, false, H / 8, a.I_sh, H / 2, 8, 128, 32))) return rc;
    if ((rc = make_map(&msu, a.su_q, false, H / 8, a.I_sh, H / 2, 8, 128, 32))) return rc;
    if ((rc = make_map(&msd, a.sd_q, false, a.I_sh / 8, H, a.I_sh / 2, 8, 128, 32))) return rc;
  } else {
    msg = msu = msd = mg;
  }

  TcArgs t;
  t.offsets = a.offsets;
  t.perm = a.perm;
  t.E = a.E;
  t.P = a.P;
  t.k = a.k > 0 ? a.k : 1;
  t.H = H;
  t.I = a.I;
  t.I_sh = a.I_sh;
  t.h = a.h;
  t.h_stride = a.h_stride;
  t.ypick = a.ypick;
  t.ep = a.ep;
  t.err = w.counts + 2;

  const int grid_gu = (int)(gu < (size_t)sm_count() ? gu : (size_t)sm_count());
  t.tiles = w.tiles_gu;
  t.ntiles = w.counts;
  t.s0 = a.g_s;
  t.b0 = a.g_b;
  t.s1 = a.u_s;
  t.b1 = a.u_b;
  t.ss0 = a.sg_s;
  t.sb0 = a.sg_b;
  t.ss1 = a.su_s;
  t.sb1 = a.su_b;
  prof_begin("experts_gateup", st);
  moe_tc_kernel<true><<<grid_gu, TC_THREADS, TC_SMEM, st>>>(ma, mg, mu, msg, msu, t);
  prof_end("experts_gateup", st);
  LG_LAUNCH_CHECK("moe_tc_gateup");

  const int grid_dn = (int)(dn < (size_t)sm_count() ? dn : (size_t)sm_count());
  t.tiles = w.tiles_dn;
  t.ntiles = w.counts + 1;
  t.s0 = a.d_s;
  t.b0 = a.d_b;
  t.s1 = a.d_s;
  t.b1 = a.d_b;
  t.ss0 = a.sd_s;
  t.sb0 = a.sd_b;
  t.ss1 = a.sd_s;
  t.sb1 = a.sd_b;
  prof_begin("experts_down", st);
  moe_tc_kernel<false><<<grid_dn, TC_THREADS, TC_SMEM, st>>>(mh, md, md, msd, msd, t);
  prof_end("experts_down", st);
  LG_LAUNCH_CHECK("moe_tc_down");
  return LG_OK;
}

// Status word of the last tensor-core launch in this workspace (0 = ok; otherwise the role
// whose bounded wait expired). Synchronous; for tests and diagnostics.
int* tc_err_word(void* tc_ws, int T, int H, int I, int I_sh, int E, int k) {
  TcWs w;
  carve_tc(tc_ws, T, H, I, I_sh, E, k, &w);
  return w.counts + 2;
}

int tc_status(const void* tc_ws, int T, int H, int I, int I_sh, int E, int k, int* status) {
  TcWs w;
  carve_tc(const_cast<void*>(tc_ws), T, H, I, I_sh, E, k, &w);
  LG_CUDA_TRY(cudaMemcpy(status, w.counts + 2, sizeof(int), cudaMemcpyDeviceToHost));
  return LG_OK;
}

#ifdef LG_TC_PROFILE
extern "C" int lg_tc_set_stats(void* p) {
  return cudaMemcpyToSymbol(g_tc_stats, &p, sizeof(p)) == cudaSuccess ? 0 : 3;
}
#endif

}  // namespace lg
