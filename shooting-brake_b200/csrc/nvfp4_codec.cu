// NVFP4 codec kernels: bit-exact dequantisation and the reference quantiser.
//
// Dequant: W[r][c] = e2m1(nibble) * fp32(e4m3(sf[r][c/16]) * g), low nibble =
// even c -- the reference CPU tier's decode (src/phase7/cpu_expert_capi.cpp:
// 301-346) and vLLM dequantize_to_dtype (the decoder the reference's tests
// trust, src/phase7/nvfp4_testutil.py:53-71).
//
// Quantise: vLLM ref_nvfp4_quant, the quantiser behind the reference's
// fixtures and the benchmark weights. Per 16-element block with quantisation
// global G (= 448*6/amax):
//   scale = clamp(G * (amax_block * fp32(1/6)), -448, 448) -> e4m3 (nearest even)
//   inv   = 1 / (fp32(e4m3) * (1 / G))
//   code  = cast_to_fp4(clamp(x * inv, -6, 6))  (nearest, ties to the even code)
// Every fp32 step uses the _rn intrinsics so no FMA contraction changes a bit.
#include <cuda_fp8.h>

#include "common.cuh"
#include "kernels.h"

namespace sbb {

namespace {

__global__ void dequant_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf,
                               const float* __restrict__ g, int64_t rows_per_scale,
                               float* __restrict__ out, int64_t rows, int64_t cols) {
  const int64_t nblk = cols / 16;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nblk) return;
  const int64_t r = idx / nblk, b = idx - r * nblk;
  const float bs = __fmul_rn(e4m3_to_float(sf[idx]), g[r / rows_per_scale]);
  const uint2 packed = *reinterpret_cast<const uint2*>(q + r * (cols / 2) + b * 8);
  float v[16];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t word = j < 4 ? packed.x : packed.y;
    const uint32_t byte = (word >> (8 * (j & 3))) & 0xFFu;
    v[2 * j] = __fmul_rn(e2m1_to_float(byte & 0xFu), bs);
    v[2 * j + 1] = __fmul_rn(e2m1_to_float(byte >> 4), bs);
  }
  float4* o = reinterpret_cast<float4*>(out + r * cols + b * 16);
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

__device__ __forceinline__ uint32_t fp4_code(float x) {
  const float a = fabsf(x);
  uint32_t m = 0;
  if (a > 0.25f && a < 0.75f) m = 1;
  else if (a >= 0.75f && a <= 1.25f) m = 2;
  else if (a > 1.25f && a < 1.75f) m = 3;
  else if (a >= 1.75f && a <= 2.5f) m = 4;
  else if (a > 2.5f && a < 3.5f) m = 5;
  else if (a >= 3.5f && a <= 5.0f) m = 6;
  else if (a > 5.0f) m = 7;
  return (x < 0.0f && m != 0) ? (m | 8u) : m;
}

__global__ void quantize_kernel(const void* __restrict__ x, int in_dt, const float* __restrict__ gq,
                                int64_t rows_per_scale, uint8_t* __restrict__ q,
                                uint8_t* __restrict__ sf, int64_t rows, int64_t cols) {
  const int64_t nblk = cols / 16;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nblk) return;
  const int64_t r = idx / nblk, b = idx - r * nblk;
  float v[16];
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = load_act(x, (size_t)(r * cols + b * 16 + j), in_dt);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  const float G = gq[r / rows_per_scale];
  float scale = __fmul_rn(G, __fmul_rn(amax, 1.0f / 6.0f));
  scale = fminf(fmaxf(scale, -448.0f), 448.0f);
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(scale, __NV_SATFINITE, __NV_E4M3);
  const float sq = e4m3_to_float(s8);
  const float inv_g = __fdiv_rn(1.0f, G == 0.0f ? __fadd_rn(G, 1e8f) : G);
  const float t = __fmul_rn(sq, inv_g);
  const float out_scale = __fdiv_rn(1.0f, t == 0.0f ? __fadd_rn(t, 1e8f) : t);
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float s = __fmul_rn(v[j], out_scale);
    s = fminf(fmaxf(s, -6.0f), 6.0f);
    const uint32_t c = fp4_code(s);
    if (j < 8) w0 |= c << (4 * j);
    else w1 |= c << (4 * (j - 8));
  }
  *reinterpret_cast<uint2*>(q + r * (cols / 2) + b * 8) = make_uint2(w0, w1);
  sf[idx] = (uint8_t)s8;
}

}  // namespace

cudaError_t launch_dequant(const uint8_t* q, const uint8_t* sf, const float* g,
                           int64_t rows_per_scale, float* out, int64_t rows, int64_t cols,
                           cudaStream_t stream) {
  const int64_t n = rows * (cols / 16);
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  dequant_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
      q, sf, g, rows_per_scale, out, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_quantize(const void* x, int in_dt, const float* gq, int64_t rows_per_scale,
                            uint8_t* q, uint8_t* sf, int64_t rows, int64_t cols,
                            cudaStream_t stream) {
  const int64_t n = rows * (cols / 16);
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  quantize_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
      x, in_dt, gq, rows_per_scale, q, sf, rows, cols);
  return cudaGetLastError();
}

}  // namespace sbb
