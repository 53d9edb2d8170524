// Top-k weighted combine: out[t, :] = sum_k w[t, k] * y[slot_of[t*top_k+k], :]
// over the token's valid routes, in ascending k, fp32 accumulation.
//
// This is the reference's deterministic combine (src/phase7/xe2_nvfp4/
// grouped_moe.cpp:481-500: per token, gather its routes through the inverse
// map and skip invalid ones by index) rather than its atomic scatter-add
// (nvfp4_moe_grouped.sycl.cpp:508-524), so a token's sum has one fixed order.
// The output is written once in the requested dtype, which also replaces the
// op's zero-fill (src/QuixiCore-XPU/src/dispatch/moe.cpp:45): tokens without a
// valid route get zeros.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace sbb {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void store4(void* out, int out_dt, int64_t at, float4 acc) {
  if (out_dt == kF32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + at) = acc;
  } else if (out_dt == kBF16) {
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + at) = u;
  } else {
    __half2 a = __floats2half2_rn(acc.x, acc.y);
    __half2 b = __floats2half2_rn(acc.z, acc.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__half*>(out) + at) = u;
  }
}

__global__ void __launch_bounds__(kThreads) combine_kernel(
    const float* __restrict__ y, const int32_t* __restrict__ slot_of,
    const float* __restrict__ weights, int multiply_router_weight, void* __restrict__ out,
    int out_dt, int top_k, int K) {
  const int64_t t = blockIdx.x;
  __shared__ int32_t s_slot[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x < top_k) {
    s_slot[threadIdx.x] = slot_of[t * top_k + threadIdx.x];
    s_w[threadIdx.x] = multiply_router_weight ? weights[t * top_k + threadIdx.x] : 1.0f;
  }
  __syncthreads();
  for (int n4 = (blockIdx.y * kThreads + threadIdx.x) * 4; n4 < K;
       n4 += gridDim.y * kThreads * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // routes in groups of 8: the group's loads are all issued before the
    // sums, which still run in ascending k
    for (int k0 = 0; k0 < top_k; k0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int32_t s = k0 + j < top_k ? s_slot[k0 + j] : -1;
        v[j] = s >= 0 ? __ldg(reinterpret_cast<const float4*>(y + (int64_t)s * K + n4))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (k0 + j >= top_k || s_slot[k0 + j] < 0) continue;
        const float w = s_w[k0 + j];
        acc.x = fmaf(w, v[j].x, acc.x);
        acc.y = fmaf(w, v[j].y, acc.y);
        acc.z = fmaf(w, v[j].z, acc.z);
        acc.w = fmaf(w, v[j].w, acc.w);
      }
    }
    store4(out, out_dt, t * K + n4, acc);
  }
}

}  // namespace

cudaError_t launch_combine(const float* y, const int32_t* slot_of, const float* weights,
                           int multiply_router_weight, void* out, int out_dt, int64_t M,
                           int top_k, int K, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  // K is a multiple of 32, so whole float4 groups cover each row.
  const int per_cta = kThreads * 4;
  dim3 grid((unsigned)M, (unsigned)((K + per_cta - 1) / per_cta));
  return launch_kernel(true, combine_kernel, grid, dim3(kThreads), 0, stream, y, slot_of, weights,
                       multiply_router_weight, out, out_dt, top_k, K);
}

}  // namespace sbb
