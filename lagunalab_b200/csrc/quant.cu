// Affine quantize / dequantize of rows in the MLX packed layout.
//
// quantize_rows_kernel: one thread per (row, group): min/max of the group, scale and bias
//   rounded to bf16, codes rint((x - bias) / scale) clamped to [0, 2^bits - 1] (IEEE division
//   and round-half-even, so results are bit-exact against a CPU restatement), packed low bits
//   first into the row's uint32 words.  Used for the KV-cache append (the role of mx.quantize
//   inside mlx-lm's QuantizedKVCache, laguna_mlx/cache.py:90) and for weight conversion.
// dequantize_rows_kernel: value = scale * code + bias -> bf16 (the DequantKVCache multi-token
//   path, laguna_mlx/cache.py:99-100).
#include <math.h>

#include "common.cuh"

namespace lg {

template <int BITS>
__global__ void quantize_rows_kernel(const void* __restrict__ x, int x_f32, int B, int H, int L,
                                     int D, long long sb, long long sh, long long sl, int group,
                                     uint32_t* __restrict__ dq, __nv_bfloat16* __restrict__ ds,
                                     __nv_bfloat16* __restrict__ dbias, int cap, int offset) {
  const int ngroups = D / group;
  const long long total = (long long)B * H * L * ngroups;
  const int per_word = 32 / BITS;
  const float nb = (float)((1 << BITS) - 1);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(i % ngroups);
    long long rr = i / ngroups;
    const int l = (int)(rr % L);
    rr /= L;
    const int h = (int)(rr % H);
    const int b = (int)(rr / H);
    const long long src = b * sb + h * sh + l * sl + (long long)g * group;
    auto ld = [&](int j) -> float {
      return x_f32 ? static_cast<const float*>(x)[src + j]
                   : bf2f(static_cast<const __nv_bfloat16*>(x)[src + j]);
    };
    float lo = INFINITY, hi = -INFINITY;
    for (int j = 0; j < group; ++j) {
      float v = ld(j);
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
    __nv_bfloat16 sbf, bbf;
    quant_group_params(lo, hi, nb, &sbf, &bbf);
    const float s = bf2f(sbf), bv = bf2f(bbf);
    const size_t row = ((size_t)b * H + h) * cap + offset + l;
    uint32_t* wrow = dq + row * (D * BITS / 32) + (size_t)g * (group * BITS / 32);
    for (int w = 0; w < group / per_word; ++w) {
      uint32_t word = 0;
      for (int j = 0; j < per_word; ++j) {
        word |= quant_code(ld(w * per_word + j), s, bv, nb) << (BITS * j);
      }
      wrow[w] = word;
    }
    ds[row * ngroups + g] = sbf;
    dbias[row * ngroups + g] = bbf;
  }
}

template <int BITS>
__global__ void dequantize_rows_kernel(const uint32_t* __restrict__ q,
                                       const __nv_bfloat16* __restrict__ s,
                                       const __nv_bfloat16* __restrict__ bb, int B, int H, int cap,
                                       int n, int D, int group, __nv_bfloat16* __restrict__ out) {
  const long long total = (long long)B * H * n * D;
  const int per_word = 32 / BITS;
  const int wpr = D * BITS / 32, gpr = D / group;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    long long rr = i / D;
    const int t = (int)(rr % n);
    const long long bh = rr / n;
    const size_t row = (size_t)bh * cap + t;
    const uint32_t w = q[row * wpr + d / per_word];
    const uint32_t c = (w >> (BITS * (d % per_word))) & ((1u << BITS) - 1u);
    const float v = fmaf(bf2f(s[row * gpr + d / group]), code_to_f(c), bf2f(bb[row * gpr + d / group]));
    out[i] = __float2bfloat16_rn(v);
  }
}

}  // namespace lg

using namespace lg;

extern "C" int lg_quantize_rows(const void* x, int x_is_f32, int B, int H, int L, int D,
                                long long sb, long long sh, long long sl, int bits,
                                int group_size, uint32_t* dst_q, void* dst_s, void* dst_b,
                                int cap, int offset, void* stream) {
  LG_CHECK_ARG(bits == 4 || bits == 8, "quantize: bits %d not in {4, 8}", bits);
  LG_CHECK_ARG(group_size == 32 || group_size == 64 || group_size == 128,
               "quantize: group_size %d not in {32, 64, 128}", group_size);
  LG_CHECK_ARG(D > 0 && D % group_size == 0, "quantize: head_dim %d is not a multiple of group_size %d",
               D, group_size);
  LG_CHECK_ARG(B >= 0 && H >= 0 && L >= 0 && offset >= 0 && offset + L <= cap,
               "quantize: rows [%d, %d) do not fit capacity %d", offset, offset + L, cap);
  LG_CHECK_ARG(x && dst_q && dst_s && dst_b, "quantize: NULL pointer");
  long long total = (long long)B * H * L * (D / group_size);
  if (total == 0) return LG_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (bits == 8)
    quantize_rows_kernel<8><<<blocks, 256, 0, st>>>(x, x_is_f32, B, H, L, D, sb, sh, sl,
                                                    group_size, dst_q,
                                                    static_cast<__nv_bfloat16*>(dst_s),
                                                    static_cast<__nv_bfloat16*>(dst_b), cap, offset);
  else
    quantize_rows_kernel<4><<<blocks, 256, 0, st>>>(x, x_is_f32, B, H, L, D, sb, sh, sl,
                                                    group_size, dst_q,
                                                    static_cast<__nv_bfloat16*>(dst_s),
                                                    static_cast<__nv_bfloat16*>(dst_b), cap, offset);
  LG_LAUNCH_CHECK("quantize_rows");
  return LG_OK;
}

extern "C" int lg_dequantize_rows(const uint32_t* q, const void* s, const void* b, int B, int H,
                                  int cap, int n, int D, int bits, int group_size, void* out,
                                  void* stream) {
  LG_CHECK_ARG(bits == 4 || bits == 8, "dequantize: bits %d not in {4, 8}", bits);
  LG_CHECK_ARG(group_size == 32 || group_size == 64 || group_size == 128,
               "dequantize: group_size %d", group_size);
  LG_CHECK_ARG(D > 0 && D % group_size == 0, "dequantize: head_dim %d / group %d", D, group_size);
  LG_CHECK_ARG(n >= 0 && n <= cap, "dequantize: n=%d cap=%d", n, cap);
  LG_CHECK_ARG(q && s && b && out, "dequantize: NULL pointer");
  long long total = (long long)B * H * n * D;
  if (total == 0) return LG_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (bits == 8)
    dequantize_rows_kernel<8><<<blocks, 256, 0, st>>>(q, static_cast<const __nv_bfloat16*>(s),
                                                      static_cast<const __nv_bfloat16*>(b), B, H,
                                                      cap, n, D, group_size,
                                                      static_cast<__nv_bfloat16*>(out));
  else
    dequantize_rows_kernel<4><<<blocks, 256, 0, st>>>(q, static_cast<const __nv_bfloat16*>(s),
                                                      static_cast<const __nv_bfloat16*>(b), B, H,
                                                      cap, n, D, group_size,
                                                      static_cast<__nv_bfloat16*>(out));
  LG_LAUNCH_CHECK("dequantize_rows");
  return LG_OK;
}
