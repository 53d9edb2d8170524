// Shared device helpers for the routed-expert NVFP4 MoE kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace sbb {

// --------------------------------------------------------------------------
// NVFP4 element and scale decode.
//
// Weight = e2m1(nibble) * e4m3(block scale) * global, low nibble = even k.
// e2m1 has 1 mantissa bit and e4m3 3, so their product has at most 6
// significant bits and lies in [2^-10, 2688] when nonzero: it is exact in
// both f16 and bf16. The per-expert fp32 global is applied to fp32 sums.
// --------------------------------------------------------------------------

__device__ __forceinline__ float e2m1_to_float(uint32_t nib) {
  // magnitude ladder {0, .5, 1, 1.5, 2, 3, 4, 6}
  const uint32_t mag = nib & 7u;
  uint32_t bits = 0x3F000000u + (mag << 22);  // 2..7 -> 1, 1.5, 2, 3, 4, 6
  bits = mag < 2u ? (mag ? 0x3F000000u : 0u) : bits;
  bits |= (nib & 8u) << 28;
  return __uint_as_float(bits);
}

__device__ __forceinline__ float e4m3_to_float(uint32_t v) {
  const uint32_t exp = (v >> 3) & 0xFu;
  const uint32_t man = v & 7u;
  float f;
  if (exp == 0u) {
    f = __int2float_rn((int)man) * 0.001953125f;  // man * 2^-9
  } else if (exp == 15u && man == 7u) {
    f = __uint_as_float(0x7FC00000u);
  } else {
    f = __uint_as_float(((exp + 120u) << 23) | (man << 20));
  }
  return (v & 0x80u) ? -f : f;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// --------------------------------------------------------------------------
// Activation dtypes, mirroring the reference op's DType {f32, f16, bf16}.
// --------------------------------------------------------------------------
enum ActType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

__device__ __forceinline__ float load_act(const void* p, size_t i, int dt) {
  if (dt == kBF16) return bf16_bits_to_float(static_cast<const uint16_t*>(p)[i]);
  if (dt == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace sbb

namespace sbb {

// --------------------------------------------------------------------------
// Cross-GPU flags (expert-parallel exchange over NVLink peer memory).
// --------------------------------------------------------------------------

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Spin until *flag (its high word when hi_word) equals epoch, or give up at
// `deadline` (globaltimer ns) or once *errors has bit 0 set (an earlier wait
// of this rank gave up), raising bit 0 of *errors. *seen gets the flag.
__device__ __forceinline__ bool ep_wait_epoch(const unsigned long long* flag,
                                              unsigned long long epoch, bool hi_word,
                                              unsigned long long* seen, unsigned int* errors,
                                              uint64_t deadline) {
  for (uint32_t i = 0;; ++i) {
    const unsigned long long v = ld_acquire_sys(flag);
    if ((hi_word ? (v >> 32) : v) == epoch) {
      *seen = v;
      return true;
    }
    if ((i & 63u) == 63u) {
      if (globaltimer_ns() > deadline || (*reinterpret_cast<volatile unsigned int*>(errors) & 1u)) {
        atomicOr(errors, 1u);
        return false;
      }
    }
  }
}

}  // namespace sbb
