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
#include "gemv_core.cuh"
#include "moe.cuh"

namespace lg {

// token (activation row) of group row j: routed picks p < P come from token p / k, shared
// rows p >= P from token p - P.
__device__ __forceinline__ int row_token(int p, int P, int k) { return p < P ? p / k : p - P; }

constexpr int GV_WARPS = 4;

__global__ void __launch_bounds__(GV_WARPS * 32) moe_gemv_gateup_kernel(GemvArgs a) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  __shared__ float red[GV_WARPS][2][32][4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int na = a.active[0];
  if ((int)blockIdx.y >= na) return;
  const int g = a.active[1 + blockIdx.y];
  const bool sh = (g == a.E);
  const int Ig = sh ? a.I_sh : a.I;
  const int m0 = blockIdx.x * 16;
  if (m0 >= Ig) return;
  const int row0 = a.offsets[g], cnt = a.offsets[g + 1] - row0;
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

  for (int tb = 0; tb < cnt; tb += 8) {
    const int tn = tb + r;  // this thread's B-fragment token (row of the group)
    const bool tval = tn < cnt;
    const int tok = tval ? row_token(a.perm[row0 + tn], a.P, a.k) : 0;
    const __nv_bfloat16* xrow = a.x + (size_t)tok * H;
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int gg = warp; gg < gpr; gg += GV_WARPS) {
      const size_t wo = (size_t)gg * 8 + 2 * c4;
      const uint2 g0 = *reinterpret_cast<const uint2*>(gq + (size_t)ra * wpr + wo);
      const uint2 g8 = *reinterpret_cast<const uint2*>(gq + (size_t)rb * wpr + wo);
      const uint2 u0 = *reinterpret_cast<const uint2*>(uq + (size_t)ra * wpr + wo);
      const uint2 u8 = *reinterpret_cast<const uint2*>(uq + (size_t)rb * wpr + wo);
      uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0;
      if (tval) {
        xa0 = *reinterpret_cast<const uint4*>(xrow + gg * 64 + 16 * c4);
        xa1 = *reinterpret_cast<const uint4*>(xrow + gg * 64 + 16 * c4 + 8);
      }
      // per-token group sum, moved from token-major (lane/4) to the C layout (cols 2c4, 2c4+1)
      float xs = xsum16(xa0, xa1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 2);
      const float xs0 = __shfl_sync(0xffffffffu, xs, (2 * c4) * 4);
      const float xs1 = __shfl_sync(0xffffffffu, xs, (2 * c4 + 1) * 4);
      const float sg0 = bf2f(gs[(size_t)ra * gpr + gg]), sg8 = bf2f(gs[(size_t)rb * gpr + gg]);
      const float bg0 = bf2f(gb[(size_t)ra * gpr + gg]), bg8 = bf2f(gb[(size_t)rb * gpr + gg]);
      const float su0 = bf2f(us[(size_t)ra * gpr + gg]), su8 = bf2f(us[(size_t)rb * gpr + gg]);
      const float bu0 = bf2f(ub[(size_t)ra * gpr + gg]), bu8 = bf2f(ub[(size_t)rb * gpr + gg]);
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
        const int col = tb + 2 * c4 + (j & 1);   // group row (token tile column)
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

__global__ void __launch_bounds__(GV_WARPS * 32) moe_gemv_down_kernel(GemvArgs a) {
  pdl_wait();  // inputs come from the previous kernel
  pdl_trigger();
  __shared__ float red[GV_WARPS][32][4];
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

  for (int tb = 0; tb < cnt; tb += 8) {
    const int tn = tb + r;
    const bool tval = tn < cnt;
    const __nv_bfloat16* hrow = a.h + (size_t)(row0 + (tval ? tn : 0)) * a.h_stride;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int gg = warp; gg < gpr; gg += GV_WARPS) {
      const size_t wo = (size_t)gg * 8 + 2 * c4;
      const uint2 w0 = *reinterpret_cast<const uint2*>(dq + (size_t)ra * wpr + wo);
      const uint2 w8 = *reinterpret_cast<const uint2*>(dq + (size_t)rb * wpr + wo);
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
      const float s0 = bf2f(ds[(size_t)ra * gpr + gg]), s8 = bf2f(ds[(size_t)rb * gpr + gg]);
      const float b0 = bf2f(db[(size_t)ra * gpr + gg]), b8 = bf2f(db[(size_t)rb * gpr + gg]);
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
        const int col = tb + 2 * c4 + (j & 1);
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

int launch_gemv(const GemvArgs& a, int max_groups, cudaStream_t s) {
  if (max_groups <= 0) return LG_OK;
  const int Imax = a.I > a.I_sh ? a.I : a.I_sh;
  dim3 g1((Imax + 15) / 16, max_groups);
  prof_begin("experts_gateup", s);
  LG_CUDA_TRY(launch_k(moe_gemv_gateup_kernel, g1, dim3(GV_WARPS * 32), 0, s, a));
  prof_end("experts_gateup", s);
  LG_LAUNCH_CHECK("moe_gemv_gateup");
  dim3 g2((a.H + 15) / 16, max_groups);
  prof_begin("experts_down", s);
  LG_CUDA_TRY(launch_k(moe_gemv_down_kernel, g2, dim3(GV_WARPS * 32), 0, s, a));
  prof_end("experts_down", s);
  LG_LAUNCH_CHECK("moe_gemv_down");
  return LG_OK;
}

}  // namespace lg
