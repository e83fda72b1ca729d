// Decoder-layer kernels around the MoE block and the decode attention, for the full Laguna
// decoder (laguna_mlx/laguna.py:75-206): RMSNorm with an optional fused residual add, the
// 4-bit dense linear as a decode-size tensor-core GEMV, the quantized token embedding, the
// attention prologue (per-head q/k RMSNorm, RoPE, bf16 KV-cache append, softplus output gate)
// and the greedy argmax. Rounding follows the MLX graph: every op output is materialised in
// bf16 and the kernels round at the same points.
#include <math.h>

#include "common.cuh"
#include "decode_core.cuh"
#include "gemv_core.cuh"
#include "prep_core.cuh"

namespace lg {

__device__ __forceinline__ uint2 ldg_stream_u2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------------------
// RMSNorm (laguna.py:158-160, :189; mx.fast.rms_norm): y = bf16(bf16(h * rsqrt(mean(h^2) +
// eps)) * w), fp32 statistics. With a residual, h = bf16(x + residual) is the decoder's
// residual stream (laguna.py:163-164) and is written out too.
// ---------------------------------------------------------------------------------------
constexpr int RN_THREADS = 256;

__global__ void __launch_bounds__(RN_THREADS) rmsnorm_kernel(const __nv_bfloat16* x,
                                                             const __nv_bfloat16* res,
                                                             const __nv_bfloat16* w, int H,
                                                             float eps, __nv_bfloat16* sum_out,
                                                             __nv_bfloat16* out) {
  extern __shared__ __align__(16) uint4 hsm[];  // the row being normalised, [H / 8]
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  const uint4* rr = res ? reinterpret_cast<const uint4*>(res + (size_t)t * H) : nullptr;
  uint4* so = sum_out ? reinterpret_cast<uint4*>(sum_out + (size_t)t * H) : nullptr;
  const int nv = H / 8;
  for (int i = threadIdx.x; i < nv; i += RN_THREADS) {
    uint4 v = xr[i];
    if (rr) {
      v = add8_bf16(v, rr[i]);
      if (so) so[i] = v;
    }
    hsm[i] = v;
  }
  __syncthreads();
  const float r = block_rms_scale(hsm, H, eps, red);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < nv; i += RN_THREADS) orow[i] = rms_apply8(hsm[i], wr[i], r);
}

// ---------------------------------------------------------------------------------------
// 4-bit dense linear at decode sizes (nn.QuantizedLinear, laguna.py:84-92, :197):
// y[t, n] = sum_k x[t, k] * (scale[n, k/64] * code[n, k] + bias[n, k/64]), fp32 accumulation,
// one bf16 rounding (quantized_matmul's output), then optionally + residual in bf16.
// One CTA per (16-row tile of W, 16 tokens), 16 warps split the K groups, each warp runs the
// tensor-core group product of gemv_core.cuh against one or two 8-token tiles.
// ---------------------------------------------------------------------------------------
constexpr int QL_WARPS = 16;
constexpr int QL_MAX_T = 64;  // tokens per call: up to four 16-token CTA rows per W tile

struct QlArgs {
  const __nv_bfloat16* x;  // [T, K]
  const uint32_t* wq;      // [N, K / 8]
  const __nv_bfloat16* ws; // [N, K / 64]
  const __nv_bfloat16* wb;
  const __nv_bfloat16* res;  // [T, N] or null
  __nv_bfloat16* out;        // [T, N]
  int T, K, N;
};

// NG: groups per warp handled per pass; the first pass's weights and scales are loaded before
// the PDL wait (weights are static), so they stream while the previous kernel finishes.
template <int NTT, int NG>
__global__ void __launch_bounds__(QL_WARPS * 32) qlinear_kernel(QlArgs a) {
  __shared__ float red[QL_WARPS][32][4 * NTT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c4 = lane & 3;
  const int m0 = blockIdx.x * 16;
  // blockIdx.y: this CTA's 16 tokens (CTAs of the same W tile share its reads through L2)
  const int t0 = blockIdx.y * 16;
  const int T = min(a.T - t0, 16);
  const __nv_bfloat16* xb = a.x + (size_t)t0 * a.K;
  const __nv_bfloat16* resb = a.res ? a.res + (size_t)t0 * a.N : nullptr;
  __nv_bfloat16* outb = a.out + (size_t)t0 * a.N;
  const int ra = min(m0 + r, a.N - 1), rb = min(m0 + r + 8, a.N - 1);
  const int K = a.K, wpr = K / 8, gpr = K / 64;
  float acc[NTT][4];
#pragma unroll
  for (int tt = 0; tt < NTT; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
  bool waited = false;
  for (int g0 = warp; g0 < gpr || !waited; g0 += NG * QL_WARPS) {
    uint2 w0[NG], w8[NG];
    float s0[NG], s8[NG], b0[NG], b8[NG];
#pragma unroll
    for (int i = 0; i < NG; ++i) {
      const int gg = g0 + i * QL_WARPS;
      if (gg < gpr) {
        const size_t wo = (size_t)gg * 8 + 2 * c4;
        w0[i] = ldg_stream_u2(a.wq + (size_t)ra * wpr + wo);
        w8[i] = ldg_stream_u2(a.wq + (size_t)rb * wpr + wo);
        s0[i] = bf2f(a.ws[(size_t)ra * gpr + gg]);
        s8[i] = bf2f(a.ws[(size_t)rb * gpr + gg]);
        b0[i] = bf2f(a.wb[(size_t)ra * gpr + gg]);
        b8[i] = bf2f(a.wb[(size_t)rb * gpr + gg]);
      }
    }
    if (!waited) {  // x comes from the previous kernel
      pdl_wait();
      pdl_trigger();
      waited = true;
    }
#pragma unroll
    for (int i = 0; i < NG; ++i) {
      const int gg = g0 + i * QL_WARPS;
      if (gg >= gpr) break;
#pragma unroll
      for (int tt = 0; tt < NTT; ++tt) {
        const int tok = 8 * tt + r;
        uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
        if (tok < T) {
          const __nv_bfloat16* xr = xb + (size_t)tok * K + gg * 64 + 16 * c4;
          xa0 = *reinterpret_cast<const uint4*>(xr);
          xa1 = *reinterpret_cast<const uint4*>(xr + 8);
        }
        float xs = xsum16(xa0, xa1);
        xs += __shfl_xor_sync(0xffffffffu, xs, 1);
        xs += __shfl_xor_sync(0xffffffffu, xs, 2);
        const float xs0 = __shfl_sync(0xffffffffu, xs, (2 * c4) * 4);
        const float xs1 = __shfl_sync(0xffffffffu, xs, (2 * c4 + 1) * 4);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        group_mma(d, w0[i], w8[i], xa0, xa1);
        acc[tt][0] += s0[i] * d[0] + b0[i] * xs0;
        acc[tt][1] += s0[i] * d[1] + b0[i] * xs1;
        acc[tt][2] += s8[i] * d[2] + b8[i] * xs0;
        acc[tt][3] += s8[i] * d[3] + b8[i] * xs1;
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < NTT; ++tt)
#pragma unroll
    for (int j = 0; j < 4; ++j) red[warp][lane][4 * tt + j] = acc[tt][j];
  __syncthreads();
  // 32 lanes x 4 NTT values: spread the cross-warp sums over the CTA's threads
  for (int i = threadIdx.x; i < 32 * 4 * NTT; i += QL_WARPS * 32) {
    const int l = i / (4 * NTT), q = i % (4 * NTT);
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < QL_WARPS; ++w) v += red[w][l][q];
    const int lr = l >> 2, lc = l & 3, tt = q / 4, j = q % 4;
    const int tok = 8 * tt + 2 * lc + (j & 1);
    const int n = m0 + lr + (j < 2 ? 0 : 8);
    if (tok < T && n < a.N) {
      float y = round_bf16(v);
      if (resb) y += bf2f(resb[(size_t)tok * a.N + n]);
      outb[(size_t)tok * a.N + n] = __float2bfloat16_rn(y);
    }
  }
}

// Staged form (2..64 tokens: batched decode steps, short prefills, for matrices with enough
// 16-row tiles to fill the GPU): one CTA per (16 tokens, 16-row tile of W), the tile staged
// into shared memory by bulk copies issued before the PDL wait (the weights are static); 4
// warps split the K groups of the staged tile and the tokens run in blocks of 8 against it,
// each block reduced across the warps and stored with the epilogue above. The CTAs of one
// tile are adjacent in launch order, so the tile crosses HBM about once; the activations come
// from L2.
constexpr int QS_WARPS = 4;
constexpr uint32_t QS_HDR = 128, QS_RED = QS_WARPS * 32 * 4 * 4;

static uint32_t qs_smem(int K) { return QS_HDR + QS_RED + tile_bytes(K); }

__global__ void __launch_bounds__(QS_WARPS * 32) qlinear_staged_kernel(QlArgs a) {
  extern __shared__ __align__(128) uint8_t qs_smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(qs_smem_raw);
  int* berr = reinterpret_cast<int*>(qs_smem_raw + 8);
  float (*red)[32][4] = reinterpret_cast<float (*)[32][4]>(qs_smem_raw + QS_HDR);
  uint8_t* tile = qs_smem_raw + QS_HDR + QS_RED;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, r = lane >> 2, c4 = lane & 3;
  // blockIdx.x: this CTA's 16 tokens (the CTAs of one tile are launched next to each other,
  // so its later copies hit L2); blockIdx.y: the 16-row tile of W
  const int m0 = blockIdx.y * 16, K = a.K, gpr = K / 64;
  const int tbeg = blockIdx.x * 16, tend = min(a.T, tbeg + 16);
  const uint32_t pitch = tile_pitch(K);
  if (threadIdx.x == 0) {
    *berr = 0;
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar, tile_bulk_bytes(K));
    tile_load_bulk(tile, a.wq, a.ws, a.wb, m0, K, bar);
  }
  pdl_wait();  // x (and the residual) come from the previous kernel
  pdl_trigger();
  __syncthreads();  // the barrier is initialised before anyone polls it
  const bool ok = __syncthreads_and(mbar_wait(bar, 0, berr, 1, 400000000LL));
  if (!ok && threadIdx.x == 0)  // the tile never arrived: drain (bounded); the rows become NaN
    for (const long long t0 = clock64(); !mbar_try_wait(bar, 0) && clock64() - t0 < 400000000LL;) {
    }
  const __nv_bfloat16* ts = reinterpret_cast<const __nv_bfloat16*>(tile + tile_sc_off(K));
  for (int t8 = tbeg; t8 < tend; t8 += 8) {
    const int tok = t8 + r;
    const bool tval = ok && tok < tend;
    const __nv_bfloat16* xr = a.x + (size_t)(tval ? tok : 0) * K;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int gg = warp; ok && gg < gpr; gg += QS_WARPS) {
      const uint32_t o0 = r * pitch + gg * 32 + c4 * 8;
      const uint2 w0 = *reinterpret_cast<const uint2*>(tile + o0);
      const uint2 w8 = *reinterpret_cast<const uint2*>(tile + o0 + 8 * pitch);
      uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
      if (tval) {
        xa0 = *reinterpret_cast<const uint4*>(xr + gg * 64 + 16 * c4);
        xa1 = *reinterpret_cast<const uint4*>(xr + gg * 64 + 16 * c4 + 8);
      }
      float xs = xsum16(xa0, xa1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 2);
      const float xs0 = __shfl_sync(0xffffffffu, xs, (2 * c4) * 4);
      const float xs1 = __shfl_sync(0xffffffffu, xs, (2 * c4 + 1) * 4);
      const int i0 = r * gpr + gg, i8 = i0 + 8 * gpr, nb = 16 * gpr;  // scales, then biases
      const float s0 = bf2f(ts[i0]), s8 = bf2f(ts[i8]);
      const float b0 = bf2f(ts[nb + i0]), b8 = bf2f(ts[nb + i8]);
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
        for (int w = 0; w < QS_WARPS; ++w) v += red[w][lane][j];
        const int col = t8 + 2 * c4 + (j & 1);
        const int n = m0 + r + (j < 2 ? 0 : 8);
        if (col < tend) {
          float y = round_bf16(v);
          if (a.res) y += bf2f(a.res[(size_t)col * a.N + n]);
          if (!ok) y = __int_as_float(0x7fc00000);
          a.out[(size_t)col * a.N + n] = __float2bfloat16_rn(y);
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// Quantized embedding lookup (nn.QuantizedEmbedding): out[t] = bf16(scale * code + bias) of
// row ids[t]. An id outside [0, V) gives a NaN row, so a bad id shows in the logits.
// ---------------------------------------------------------------------------------------
__global__ void embed_kernel(const int32_t* ids, const uint32_t* wq, const __nv_bfloat16* ws,
                             const __nv_bfloat16* wb, int V, int H, __nv_bfloat16* out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < V;
  const int wpr = H / 8, gpr = H / 64;
  for (int i = threadIdx.x; i < wpr; i += blockDim.x) {
    __align__(16) __nv_bfloat16 o[8];
    if (ok) {
      const uint32_t w = wq[(size_t)id * wpr + i];
      const int g = (8 * i) / 64;
      const float s = bf2f(ws[(size_t)id * gpr + g]), b = bf2f(wb[(size_t)id * gpr + g]);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(s * (float)((w >> (4 * j)) & 15u) + b);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(__int_as_float(0x7fc00000));
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * H + 8 * i) = *reinterpret_cast<uint4*>(o);
  }
}

// One warp per (token, head slot), four slots a CTA: grid x tokens, y slot quads (prep_head).
__global__ void __launch_bounds__(128) attn_prep_kernel(PrepArgs a) {
  __shared__ __align__(16) uint8_t sb[4][256];  // each warp's k/v code bytes
  pdl_wait();
  pdl_trigger();
  const int w = threadIdx.x >> 5, slot = (int)blockIdx.y * 4 + w;
  if (slot < a.Hq + 2 * a.Hkv) prep_head(a, blockIdx.x, slot, true, sb[w]);
}

// ---------------------------------------------------------------------------------------
// Greedy argmax over bf16 logits (first index among equal maxima); optionally advances a
// device-side position counter, so a whole decode step can run without the host.
// ---------------------------------------------------------------------------------------
constexpr int AM_THREADS = 1024;

__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const __nv_bfloat16* logits, int V,
                                                            int32_t* ids, int32_t* pos, int inc) {
  __shared__ float sv[AM_THREADS / 32];
  __shared__ int si[AM_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const __nv_bfloat16* row = logits + (size_t)t * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += AM_THREADS) {
    const float v = bf2f(row[i]);
    if (v > best) {  // NaN never wins
      best = v;
      bi = i;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = sv[lane];
    bi = si[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      ids[t] = bi == 0x7fffffff ? 0 : bi;
      if (pos && t == 0) pos[0] += inc;
    }
  }
}

}  // namespace lg

using namespace lg;

extern "C" int lg_rmsnorm(const void* x, const void* residual, const void* w, int T, int H,
                          float eps, void* sum_out, void* out, void* stream) {
  LG_CHECK_ARG(T >= 0 && H > 0 && H % 8 == 0 && H <= 16384,
               "rmsnorm: need H %% 8 == 0 and H <= 16384 (H=%d, T=%d)", H, T);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(x && w && out, "rmsnorm: NULL pointer");
  LG_CHECK_ARG(aligned(x, 16) && aligned(w, 16) && aligned(out, 16) &&
                   (!residual || aligned(residual, 16)) && (!sum_out || aligned(sum_out, 16)),
               "rmsnorm: tensors must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LG_CUDA_TRY(launch_k(rmsnorm_kernel, dim3(T), dim3(RN_THREADS), (size_t)H * 2, st,
                       static_cast<const __nv_bfloat16*>(x),
                       static_cast<const __nv_bfloat16*>(residual),
                       static_cast<const __nv_bfloat16*>(w), H, eps,
                       residual ? static_cast<__nv_bfloat16*>(sum_out) : nullptr,
                       static_cast<__nv_bfloat16*>(out)));
  LG_LAUNCH_CHECK("rmsnorm");
  return LG_OK;
}

extern "C" int lg_qlinear(const void* x, int T, int K, int N, const uint32_t* w_q,
                          const void* w_s, const void* w_b, int group_size, int bits,
                          const void* residual, void* out, void* stream) {
  LG_CHECK_ARG(bits == 4 && group_size == 64, "qlinear: 4-bit group-64 weights only");
  LG_CHECK_ARG(T >= 0 && T <= QL_MAX_T, "qlinear: decode sizes only (T=%d > %d: dequantize instead)",
               T, QL_MAX_T);
  LG_CHECK_ARG(K > 0 && K % 64 == 0 && N > 0, "qlinear: need K %% 64 == 0 (K=%d, N=%d)", K, N);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(x && w_q && w_s && w_b && out, "qlinear: NULL pointer");
  LG_CHECK_ARG(aligned(x, 16) && aligned(w_q, 8), "qlinear: x 16-byte, weights 8-byte aligned");
  QlArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.wq = w_q;
  a.ws = static_cast<const __nv_bfloat16*>(w_s);
  a.wb = static_cast<const __nv_bfloat16*>(w_b);
  a.res = static_cast<const __nv_bfloat16*>(residual);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.T = T;
  a.K = K;
  a.N = N;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  // the staged form when it has CTAs to fill the GPU (small matrices keep the 16-warp form)
  const int ctas = (N / 16) * ((T + 15) / 16);
  if (T >= 2 && N % 16 == 0 && ctas >= 2 * device_sm_count() && al16(w_q) && al16(w_s) &&
      al16(w_b)) {
    const uint32_t smem = qs_smem(K);
    if (smem > 48u * 1024u)
      LG_CUDA_TRY(cudaFuncSetAttribute(qlinear_staged_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    prof_begin("qlinear", st);
    LG_CUDA_TRY(launch_k(qlinear_staged_kernel, dim3((T + 15) / 16, N / 16), dim3(QS_WARPS * 32),
                         smem, st, a));
    prof_end("qlinear", st);
    LG_LAUNCH_CHECK("qlinear_staged");
    return LG_OK;
  }
  const dim3 grid((N + 15) / 16, (T + 15) / 16);
  prof_begin("qlinear", st);
  const int gpw = (K / 64 + QL_WARPS - 1) / QL_WARPS;  // groups per warp
  cudaError_t e;
  if (T <= 8)
    e = gpw <= 2 ? launch_k(qlinear_kernel<1, 2>, grid, dim3(QL_WARPS * 32), 0, st, a)
        : gpw <= 4 ? launch_k(qlinear_kernel<1, 4>, grid, dim3(QL_WARPS * 32), 0, st, a)
                   : launch_k(qlinear_kernel<1, 8>, grid, dim3(QL_WARPS * 32), 0, st, a);
  else
    e = gpw <= 2 ? launch_k(qlinear_kernel<2, 2>, grid, dim3(QL_WARPS * 32), 0, st, a)
        : gpw <= 4 ? launch_k(qlinear_kernel<2, 4>, grid, dim3(QL_WARPS * 32), 0, st, a)
                   : launch_k(qlinear_kernel<2, 8>, grid, dim3(QL_WARPS * 32), 0, st, a);
  LG_CUDA_TRY(e);
  prof_end("qlinear", st);
  LG_LAUNCH_CHECK("qlinear");
  return LG_OK;
}

extern "C" int lg_embed(const int32_t* ids, int T, const uint32_t* w_q, const void* w_s,
                        const void* w_b, int V, int H, int group_size, int bits, void* out,
                        void* stream) {
  LG_CHECK_ARG(bits == 4 && group_size == 64, "embed: 4-bit group-64 table only");
  LG_CHECK_ARG(T >= 0 && V > 0 && H > 0 && H % 64 == 0, "embed: need H %% 64 == 0 (H=%d)", H);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(ids && w_q && w_s && w_b && out && aligned(out, 16), "embed: NULL or misaligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LG_CUDA_TRY(launch_k(embed_kernel, dim3(T), dim3(128), 0, st, ids, w_q,
                       static_cast<const __nv_bfloat16*>(w_s),
                       static_cast<const __nv_bfloat16*>(w_b), V, H,
                       static_cast<__nv_bfloat16*>(out)));
  LG_LAUNCH_CHECK("embed");
  return LG_OK;
}

static int attn_prep_run(const void* qkvg, int T, int Hq, int Hkv, int D, const void* qn_w,
                         const void* kn_w, float eps, float rope_theta, const int32_t* pos_dev,
                         int pos_host, int gate_per_head, void* q_out, void* k_cache,
                         void* v_cache, const uint32_t* const* q8, const void* const* q8sb,
                         int cap, void* gate_out, const float* inv_freq, int rot_dims,
                         float mscale, int ring, int row0, void* stream, int streams = 0) {
  LG_CHECK_ARG(D % 64 == 0 && D <= 256 && Hq > 0 && Hkv > 0 && T >= 0,
               "attn_prep: head_dim %d (need a multiple of 64, <= 256)", D);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(qkvg && qn_w && kn_w && q_out && ((k_cache && v_cache) || q8) && gate_out,
               "attn_prep: NULL pointer");
  LG_CHECK_ARG(pos_dev || ring > 0 ||
                   (pos_host - row0 >= 0 && pos_host - row0 + (streams ? 1 : T) <= cap),
               "attn_prep: positions %d..%d beyond the cache rows %d..%d", pos_host,
               pos_host + T - 1, row0, row0 + cap - 1);
  LG_CHECK_ARG(ring == 0 || ring == cap, "attn_prep: a ring buffer has %d rows, not %d", cap,
               ring);
  PrepArgs a = {};
  if (int rc = prep_extend(&a, D, inv_freq, rot_dims, mscale, ring, row0, "attn_prep")) return rc;
  a.qkvg = static_cast<const __nv_bfloat16*>(qkvg);
  a.qn_w = static_cast<const __nv_bfloat16*>(qn_w);
  a.kn_w = static_cast<const __nv_bfloat16*>(kn_w);
  a.pos_dev = pos_dev;
  a.pos_host = pos_host;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.cap = cap;
  a.gate_per_head = gate_per_head;
  a.streams = streams;
  a.eps = eps;
  a.log2_theta = log2f(rope_theta);
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.gate_out = static_cast<__nv_bfloat16*>(gate_out);
  a.kq = q8 ? const_cast<uint32_t*>(q8[0]) : nullptr;
  a.vq = q8 ? const_cast<uint32_t*>(q8[1]) : nullptr;
  a.ks = q8 ? static_cast<__nv_bfloat16*>(const_cast<void*>(q8sb[0])) : nullptr;
  a.kb = q8 ? static_cast<__nv_bfloat16*>(const_cast<void*>(q8sb[1])) : nullptr;
  a.vs = q8 ? static_cast<__nv_bfloat16*>(const_cast<void*>(q8sb[2])) : nullptr;
  a.vb = q8 ? static_cast<__nv_bfloat16*>(const_cast<void*>(q8sb[3])) : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(T, (Hq + 2 * Hkv + 3) / 4);  // tokens on x: prefill lengths beyond 65,535
  LG_CUDA_TRY(launch_k(attn_prep_kernel, grid, dim3(128), 0, st, a));
  LG_LAUNCH_CHECK("attn_prep");
  return LG_OK;
}

extern "C" int lg_attn_prep(const void* qkvg, int T, int Hq, int Hkv, int D, const void* qn_w,
                            const void* kn_w, float eps, float rope_theta, const int32_t* pos_dev,
                            int pos_host, int gate_per_head, void* q_out, void* k_cache,
                            void* v_cache, int cap, void* gate_out, const float* inv_freq,
                            int rot_dims, float mscale, int ring, int row0, void* stream) {
  LG_CHECK_ARG(k_cache && v_cache, "attn_prep: NULL cache");
  return attn_prep_run(qkvg, T, Hq, Hkv, D, qn_w, kn_w, eps, rope_theta, pos_dev, pos_host,
                       gate_per_head, q_out, k_cache, v_cache, nullptr, nullptr, cap, gate_out,
                       inv_freq, rot_dims, mscale, ring, row0, stream);
}

extern "C" int lg_attn_prep_q8(const void* qkvg, int T, int Hq, int Hkv, int D, const void* qn_w,
                               const void* kn_w, float eps, float rope_theta,
                               const int32_t* pos_dev, int pos_host, int gate_per_head,
                               void* q_out, uint32_t* k_q, void* k_s, void* k_b, uint32_t* v_q,
                               void* v_s, void* v_b, int cap, void* gate_out,
                               const float* inv_freq, int rot_dims, float mscale, int ring,
                               int row0, void* stream) {
  LG_CHECK_ARG(k_q && k_s && k_b && v_q && v_s && v_b, "attn_prep_q8: NULL cache");
  LG_CHECK_ARG(D <= 256, "attn_prep_q8: head_dim %d > 256", D);
  const uint32_t* q8[2] = {k_q, v_q};
  const void* sb[4] = {k_s, k_b, v_s, v_b};
  return attn_prep_run(qkvg, T, Hq, Hkv, D, qn_w, kn_w, eps, rope_theta, pos_dev, pos_host,
                       gate_per_head, q_out, nullptr, nullptr, q8, sb, cap, gate_out, inv_freq,
                       rot_dims, mscale, ring, row0, stream);
}

extern "C" int lg_attn_prep_streams(const void* qkvg, int B, int Hq, int Hkv, int D,
                                    const void* qn_w, const void* kn_w, float eps,
                                    float rope_theta, const int32_t* pos_dev, int gate_per_head,
                                    void* q_out, void* k_cache, void* v_cache, int cap,
                                    void* gate_out, const float* inv_freq, int rot_dims,
                                    float mscale, int ring, void* stream) {
  LG_CHECK_ARG(k_cache && v_cache && pos_dev, "attn_prep_streams: NULL cache or positions");
  return attn_prep_run(qkvg, B, Hq, Hkv, D, qn_w, kn_w, eps, rope_theta, pos_dev, 0,
                       gate_per_head, q_out, k_cache, v_cache, nullptr, nullptr, cap, gate_out,
                       inv_freq, rot_dims, mscale, ring, 0, stream, 1);
}

extern "C" int lg_argmax(const void* logits, int T, int V, int32_t* ids, int32_t* pos, int inc,
                         void* stream) {
  LG_CHECK_ARG(T >= 0 && V > 0, "argmax: bad sizes T=%d V=%d", T, V);
  if (T == 0) return LG_OK;
  LG_CHECK_ARG(logits && ids, "argmax: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LG_CUDA_TRY(launch_k(argmax_kernel, dim3(T), dim3(AM_THREADS), 0, st,
                       static_cast<const __nv_bfloat16*>(logits), V, ids, pos, inc));
  LG_LAUNCH_CHECK("argmax");
  return LG_OK;
}
