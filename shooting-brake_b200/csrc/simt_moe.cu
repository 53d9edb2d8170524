// CUDA-core grouped expert kernels: the general-shape path (any K, I that are
// multiples of 32, every activation dtype the reference op accepts).
//
// Work is grouped by expert like the reference's grouped kernel
// (nvfp4_moe_grouped.sycl.cpp:269-405 gate/up + SwiGLU, :416-527 down), so an
// expert's weights stream from HBM once per call rather than once per route.
// One CTA owns kRows weight rows of one expert and walks that expert's routes
// in chunks of up to kTok tokens staged in shared memory as fp32. Each warp
// reduces one weight row (gate and up rows together for the first GEMM) with
// lanes striding over 32-element chunks, the decode shape of
// nvfp4_moe.sycl.cpp:66-118. Accumulation is fp32 throughout; the per-expert
// global scale multiplies the fp32 sum (nvfp4_moe_grouped.sycl.cpp:397-401).
#include "common.cuh"
#include "kernels.h"

namespace sbb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarpsPerCta = kThreads / 32;
constexpr int kRows = 32;      // weight rows (or gate/up row pairs) per CTA
constexpr int kTokMax = 8;     // tokens per staged chunk

struct Chunk32 {
  uint4 q;        // 32 packed e2m1 elements
  float s0, s1;   // block scales of elements [0,16) and [16,32)
};

__device__ __forceinline__ Chunk32 load_chunk(const uint8_t* row_q, const uint8_t* row_s, int c) {
  Chunk32 ch;
  ch.q = *reinterpret_cast<const uint4*>(row_q + (size_t)c * 16);
  ch.s0 = e4m3_to_float(row_s[2 * c]);
  ch.s1 = e4m3_to_float(row_s[2 * c + 1]);
  return ch;
}

// dot of 32 decoded elements with 32 fp32 activations; returns
// (elements 0..15 sum) * s0 + (16..31 sum) * s1.
__device__ __forceinline__ float chunk_dot(const Chunk32& ch, const float* x) {
  const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
  float part[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float acc = 0.0f;
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      const uint32_t word = w[half * 2 + wi];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        acc = fmaf(e2m1_to_float((word >> (4 * n)) & 0xFu), x[half * 16 + wi * 8 + n], acc);
      }
    }
    part[half] = acc;
  }
  return part[0] * ch.s0 + part[1] * ch.s1;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

__global__ void __launch_bounds__(kThreads) gateup_simt_kernel(
    const void* __restrict__ hidden, int act_dt, int top_k, const uint8_t* __restrict__ w13,
    const uint8_t* __restrict__ s13, const float* __restrict__ g13,
    const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ sorted, float* __restrict__ h, int K, int I, int tok_chunk) {
  extern __shared__ float s_x[];  // [tok_chunk, K]
  const int e = blockIdx.y;
  const int count = counts[e];
  if (count == 0) return;
  const int base = offsets[e];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const size_t qstride = (size_t)K / 2, sstride = (size_t)K / 16;
  const uint8_t* eq = w13 + (size_t)e * 2 * I * qstride;
  const uint8_t* es = s13 + (size_t)e * 2 * I * sstride;
  const float gs = g13[e];
  const int nchunk = K / 32;

  for (int t0 = 0; t0 < count; t0 += tok_chunk) {
    const int nt = min(tok_chunk, count - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * K; i += kThreads) {
      const int t = i / K, k = i - t * K;
      const int route = sorted[base + t0 + t];
      const size_t token = (size_t)(route / top_k);
      s_x[t * K + k] = load_act(hidden, token * K + k, act_dt);
    }
    __syncthreads();
    for (int rr = warp; rr < kRows; rr += kWarpsPerCta) {
      const int row = blockIdx.x * kRows + rr;
      if (row >= I) break;
      const uint8_t* gq = eq + (size_t)row * qstride;
      const uint8_t* gsf = es + (size_t)row * sstride;
      const uint8_t* uq = eq + (size_t)(row + I) * qstride;
      const uint8_t* usf = es + (size_t)(row + I) * sstride;
      float accg[kTokMax], accu[kTokMax];
#pragma unroll
      for (int t = 0; t < kTokMax; ++t) accg[t] = accu[t] = 0.0f;
      for (int c = lane; c < nchunk; c += 32) {
        const Chunk32 cg = load_chunk(gq, gsf, c);
        const Chunk32 cu = load_chunk(uq, usf, c);
#pragma unroll
        for (int t = 0; t < kTokMax; ++t) {
          if (t < nt) {
            accg[t] += chunk_dot(cg, s_x + t * K + c * 32);
            accu[t] += chunk_dot(cu, s_x + t * K + c * 32);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kTokMax; ++t) {
        if (t < nt) {
          const float gv = warp_sum(accg[t]) * gs;
          const float uv = warp_sum(accu[t]) * gs;
          if (lane == 0) h[(size_t)(base + t0 + t) * I + row] = silu(gv) * uv;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) down_simt_kernel(
    const float* __restrict__ h, const uint8_t* __restrict__ w2, const uint8_t* __restrict__ s2,
    const float* __restrict__ g2, const int32_t* __restrict__ counts,
    const int32_t* __restrict__ offsets, float* __restrict__ y, int K, int I, int tok_chunk) {
  extern __shared__ float s_h[];  // [tok_chunk, I]
  const int e = blockIdx.y;
  const int count = counts[e];
  if (count == 0) return;
  const int base = offsets[e];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const size_t qstride = (size_t)I / 2, sstride = (size_t)I / 16;
  const uint8_t* eq = w2 + (size_t)e * K * qstride;
  const uint8_t* es = s2 + (size_t)e * K * sstride;
  const float gs = g2[e];
  const int nchunk = I / 32;

  for (int t0 = 0; t0 < count; t0 += tok_chunk) {
    const int nt = min(tok_chunk, count - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * I; i += kThreads)
      s_h[i] = h[(size_t)(base + t0) * I + i];
    __syncthreads();
    for (int rr = warp; rr < kRows; rr += kWarpsPerCta) {
      const int row = blockIdx.x * kRows + rr;
      if (row >= K) break;
      const uint8_t* q = eq + (size_t)row * qstride;
      const uint8_t* sf = es + (size_t)row * sstride;
      float acc[kTokMax];
#pragma unroll
      for (int t = 0; t < kTokMax; ++t) acc[t] = 0.0f;
      for (int c = lane; c < nchunk; c += 32) {
        const Chunk32 ch = load_chunk(q, sf, c);
#pragma unroll
        for (int t = 0; t < kTokMax; ++t)
          if (t < nt) acc[t] += chunk_dot(ch, s_h + t * I + c * 32);
      }
#pragma unroll
      for (int t = 0; t < kTokMax; ++t) {
        if (t < nt) {
          const float v = warp_sum(acc[t]) * gs;
          if (lane == 0) y[(size_t)(base + t0 + t) * K + row] = v;
        }
      }
    }
  }
}

int tok_chunk_for(int width) {
  // keep the staged fp32 rows within 96 KB of shared memory
  int t = 24576 / width;
  return t < 1 ? 1 : (t > kTokMax ? kTokMax : t);
}

cudaError_t set_smem(const void* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

cudaError_t launch_gateup_simt(const void* hidden, int act_dt, int top_k, const uint8_t* w13,
                               const uint8_t* s13, const float* g13, const int32_t* counts,
                               const int32_t* offsets, const int32_t* sorted, float* h, int E,
                               int K, int I, cudaStream_t stream) {
  const int tc = tok_chunk_for(K);
  const size_t smem = sizeof(float) * (size_t)tc * K;
  cudaError_t err = set_smem((const void*)gateup_simt_kernel, smem);
  if (err != cudaSuccess) return err;
  dim3 grid((I + kRows - 1) / kRows, E);
  gateup_simt_kernel<<<grid, kThreads, smem, stream>>>(hidden, act_dt, top_k, w13, s13, g13,
                                                       counts, offsets, sorted, h, K, I, tc);
  return cudaGetLastError();
}

cudaError_t launch_down_simt(const float* h, const uint8_t* w2, const uint8_t* s2,
                             const float* g2, const int32_t* counts, const int32_t* offsets,
                             float* y, int E, int K, int I, cudaStream_t stream) {
  const int tc = tok_chunk_for(I);
  const size_t smem = sizeof(float) * (size_t)tc * I;
  cudaError_t err = set_smem((const void*)down_simt_kernel, smem);
  if (err != cudaSuccess) return err;
  dim3 grid((K + kRows - 1) / kRows, E);
  down_simt_kernel<<<grid, kThreads, smem, stream>>>(h, w2, s2, g2, counts, offsets, y, K, I, tc);
  return cudaGetLastError();
}

}  // namespace sbb
