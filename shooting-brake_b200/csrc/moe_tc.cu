// tcgen05 grouped expert GEMMs for the routed-expert NVFP4 MoE (sm_100a).
//
// One persistent kernel template serves both projections of every expert:
//
//   gate/up  D_g = W_gate x^T, D_u = W_up x^T   ->  h = silu(g) * u   (bf16)
//   down     D   = W2 h^T                      ->  y = D * g2          (fp32)
//
// "Swap-AB": the weights are the 128-row MMA M operand and the routed tokens
// of one expert are the N operand (N = BN in {16..128}), so a decode batch of
// 1-8 tokens per expert still runs full 128-row MMAs and a prefill batch reuses
// each dequantised weight tile across BN tokens.
//
// Work unit = (expert, token tile, weight-row tile). The units of all experts
// form one list that a grid of one CTA per SM walks round-robin (the reference
// launches one work-group per 32-row block of the sorted routes,
// nvfp4_moe_grouped.sycl.cpp:269-405; here a unit is a weight tile instead, so
// each expert's weights stream from HBM once per token tile).
//
// Warp roles of a CTA (16 warps):
//   warp 0       TMA producer: per K stage of 256, the packed e2m1 weight rows
//                (128-byte swizzle), their e4m3 scales and the token tile.
//   warp 1       TMEM allocator and MMA issuer (one thread): tcgen05.mma
//                kind::f16 with A from tensor memory and B from shared memory.
//   warps 4-11   dequant: each thread owns one weight row, turns its packed
//                bytes into exact 16-bit values e2m1 * e4m3 (the product has
//                <= 6 significant bits) and stores them straight into tensor
//                memory (tcgen05.st), where the MMA reads the A operand. The
//                dequantised tile never touches shared memory.
//   warps 12-15  epilogue: tcgen05.ld of the fp32 accumulators, global scale,
//                SwiGLU (gate/up) or the fp32 route output (down).
//
// The per-expert global scale multiplies the fp32 accumulator, as in the
// reference's grouped kernel (nvfp4_moe_grouped.sycl.cpp:397-401, 509-523),
// so the staged weight operand stays exact. Gate/up uses f16 operands: the
// gather kernel scales every activation row by a power of two into f16 range
// (exact for bf16/f16 inputs) and the epilogue multiplies it back. Down uses
// bf16 operands because h has no a-priori range bound.
//
// Tensor memory (512 columns): a ring of four A slots of 64 columns (one
// 128-row block x 128 K elements) at [0, 256) and two accumulator buffers of
// 128 columns at [256, 512). MMAs that accumulate into the same tile
// serialise on the tensor-core pipeline latency, which at N = 16 costs far
// more than the MMA itself, so consecutive K steps rotate over P independent
// partial accumulators (P = 64/BN for gate/up, whose gate and up chains also
// interleave, and 128/BN for down) that the epilogue sums.
//
// Every wait is an mbarrier try-wait loop with a deadline; on timeout the
// kernel raises status[1], drains its own in-flight copies and MMAs, frees
// its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace sbb {

namespace {

using namespace ptx;

constexpr int kBK = 256;             // K elements per pipeline stage
constexpr int kRowBytes = kBK / 2;   // packed bytes per weight row per stage (128)
constexpr int kRowScales = kBK / 16; // scale bytes per weight row per stage (16)
constexpr int kM = 128;              // MMA M
constexpr int kThreads = 512;
constexpr int kSlotCols = 64;        // TMEM columns of one A slot (128 K elements)
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr int kMaxUnitsE = kMaxExperts;

enum : int { kGateUp = 0, kDown = 1 };

struct TcParams {
  const int32_t* counts;
  const int32_t* offsets;
  const float* gscale;  // per-expert global multiplier (g13 or g2)
  const float* xscale;  // per-slot power-of-two activation scale (gate/up)
  void* out;            // gate/up: bf16 h [R, I]; down: fp32 y [R, K]
  uint32_t* status;     // status[1] |= 1 when a wait timed out
  int E;
  int I;                // intermediate size
  int m_tiles;          // weight-row tiles per expert: I/128 (gate/up), K/128 (down)
  int k_stages;         // reduction / kBK
  int rows_per_expert;  // rows of one expert in the 2-D weight maps: 2I or K
  int out_ld;           // leading dimension of out: I or K
};

template <int MODE, int BN>
struct Cfg {
  static constexpr int kNA = MODE == kGateUp ? 2 : 1;          // 128-row A blocks per stage
  static constexpr int kAStage = kNA * kM * kRowBytes;           // packed weights
  static constexpr int kSStage = kNA * kM * kRowScales;          // scales
  static constexpr int kBStage = BN * kBK * 2;                   // 16-bit tokens
  static constexpr int kStageBytes = kAStage + kBStage + kSStage;
  static constexpr int kStagesRaw = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  // A-slot uses per stage: (128-row block, K half) pairs. Even uses belong to
  // dequant warpgroup 0, odd ones to warpgroup 1.
  static constexpr int kUsesPerStage = 2 * kNA;
  // Partial accumulators per output and accumulator buffers; what they leave
  // of tensor memory forms the A ring (at most 8 slots).
  static constexpr int kP = MODE == kGateUp ? (BN <= 16 ? 2 : 1) : (BN <= 16 ? 4 : (BN <= 32 ? 2 : 1));
  static constexpr int kDBufs = 2;
  static constexpr int kOutCols = kP * BN;                             // one output (gate, up or y)
  static constexpr int kDCols = (MODE == kGateUp ? 2 : 1) * kOutCols;  // one buffer
  static constexpr int kDCol0 = kTmemCols - kDBufs * kDCols;
  static constexpr int kSlotsRaw = kDCol0 / kSlotCols;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static constexpr uint32_t kIdesc = idesc_f16(MODE == kGateUp ? 0u : 1u, kM, BN);
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kSlots >= 2, "accumulators leave no room for an A ring");
  static_assert(kStageBytes * 2 + 1024 <= 227 * 1024, "two stages must fit");
};

__device__ __forceinline__ void decode_unit(int u, int m_tiles, const int* prefix, int E, int& e,
                                            int& nt, int& mt) {
  const int t = u / m_tiles;
  mt = u - t * m_tiles;
  int lo = 0, hi = E;  // largest e with prefix[e] <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  e = lo;
  nt = t - prefix[e];
}

// Warp-uniform bounded wait: every lane polls, the warp leaves together.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  for (uint32_t i = 0;; ++i) {
    const bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    if ((i & 15) == 15) {
      int stop = 0;
      if (lane == 0) {
        stop = *abort || now_ns() > deadline;
        if (stop) *abort = 1;
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

// 128 packed elements (64 bytes, 8 scale blocks) of one row -> 64 TMEM columns
// of exact f16 pairs e2m1 * e4m3.
__device__ __forceinline__ void dequant_f16(const uint4* qv, uint2 sc, uint32_t* r) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t sp = c < 2 ? (sc.x >> (16 * c)) : (sc.y >> (16 * (c - 2)));
    const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(sp & 0xFFFFu));
    const uint32_t s0 = __byte_perm(s01, 0, 0x1010);
    const uint32_t s1 = __byte_perm(s01, 0, 0x3232);
    const uint32_t w[4] = {qv[c].x, qv[c].y, qv[c].z, qv[c].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t h[4];
      e2m1x8_to_f16x2x4(w[k], h);
      const uint32_t s = k < 2 ? s0 : s1;
#pragma unroll
      for (int b = 0; b < 4; ++b) r[16 * c + 4 * k + b] = hmul2_f16(h[b], s);
    }
  }
}

// Same for bf16 operands. The f16 pattern of an e2m1 value v, shifted right
// by 3 with the sign kept, is the bf16 pattern of v * 2^-112 (both formats
// only differ in exponent width and bias here); the block scale is staged as
// bf16(e4m3 * 2^112), so the product is exactly v * e4m3.
__device__ __forceinline__ void dequant_bf16(const uint4* qv, uint2 sc, uint32_t* r) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t sp = c < 2 ? (sc.x >> (16 * c)) : (sc.y >> (16 * (c - 2)));
    const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(sp & 0xFFFFu));
    const __half2 hs = *reinterpret_cast<const __half2*>(&s01);
    const __nv_bfloat16 b0 = __float2bfloat16_rn(__low2float(hs) * 0x1p112f);
    const __nv_bfloat16 b1 = __float2bfloat16_rn(__high2float(hs) * 0x1p112f);
    const uint32_t u0 = *reinterpret_cast<const uint16_t*>(&b0);
    const uint32_t u1 = *reinterpret_cast<const uint16_t*>(&b1);
    const uint32_t s0 = u0 | (u0 << 16);
    const uint32_t s1 = u1 | (u1 << 16);
    const uint32_t w[4] = {qv[c].x, qv[c].y, qv[c].z, qv[c].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t h[4];
      e2m1x8_to_f16x2x4(w[k], h);
      const uint32_t s = k < 2 ? s0 : s1;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t v = h[b];
        const uint32_t bf = ((v & 0x7FFF7FFFu) >> 3) | (v & 0x80008000u);
        r[16 * c + 4 * k + b] = hmul2_bf16(bf, s);
      }
    }
  }
}

template <int MODE, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmS,
                       const __grid_constant__ CUtensorMap tmB, const TcParams p) {
  using C = Cfg<MODE, BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr int NS = C::kSlots;
  __shared__ __align__(8) uint64_t full[S], empty[S], afull[NS], aempty[NS], dfull[C::kDBufs],
      dempty[C::kDBufs], done_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ int prefix[kMaxUnitsE + 1];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint64_t deadline = now_ns() + kTimeoutNs;
  volatile int* abort = &abort_s;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 8 + 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < C::kDBufs; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    mbar_init(&done_bar, 1);
    abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmS);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) {  // token-tile prefix over experts
    int carry = 0;
    for (int e0 = 0; e0 < p.E; e0 += 32) {
      const int e = e0 + lane;
      int v = e < p.E ? (p.counts[e] + BN - 1) / BN : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += n;
      }
      if (e < p.E) prefix[e + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  const int total_units = prefix[p.E] * p.m_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[S];
      bool issued[S];
#pragma unroll
      for (int i = 0; i < S; ++i) issued[i] = false;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int e, nt, mt;
        decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
        const int row_b = p.offsets[e] + nt * BN;
        for (int kk = 0; kk < p.k_stages; ++kk) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort, deadline)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::kStageBytes;
          mbar_expect_tx(&full[s], C::kStageBytes);
          const int xa = kk * kRowBytes;
          const int xs = kk * kRowScales;
          if (MODE == kGateUp) {
            const int r0 = e * p.rows_per_expert + mt * kM;
            tma_load_2d_hint(st, &tmA, &full[s], xa, r0, pol_w);
            tma_load_2d_hint(st + kM * kRowBytes, &tmA, &full[s], xa, r0 + p.I, pol_w);
            uint8_t* ss = st + C::kAStage + C::kBStage;
            tma_load_2d_hint(ss, &tmS, &full[s], xs, r0, pol_w);
            tma_load_2d_hint(ss + kM * kRowScales, &tmS, &full[s], xs, r0 + p.I, pol_w);
          } else {
            const int r0 = e * p.rows_per_expert + mt * kM;
            tma_load_2d_hint(st, &tmA, &full[s], xa, r0, pol_w);
            tma_load_2d_hint(st + C::kAStage + C::kBStage, &tmS, &full[s], xs, r0, pol_w);
          }
#pragma unroll
          for (int j = 0; j < kBK / 64; ++j)
            tma_load_2d_hint(st + C::kAStage + j * BN * 128, &tmB, &full[s], kk * kBK + j * 64,
                             row_b, pol_x);
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Never leave with copies in flight into this CTA's shared memory.
      const uint64_t drain_deadline = now_ns() + kTimeoutNs;
      for (int i = 0; i < S; ++i) {
        if (!issued[i]) continue;
        while (!mbar_try_wait(&full[i], issued_phase[i]) && now_ns() < drain_deadline) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int slot = 0;         // A ring position
      uint32_t sph = 0;     // A ring phase
      uint32_t ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++ui) {
        const int d = ui % C::kDBufs;
        if (!mbar_wait(&dempty[d], ((ui / C::kDBufs) & 1u) ^ 1u, abort, deadline)) break;
        tc_fence_after();
        const uint32_t d_tm = tmem + C::kDCol0 + d * C::kDCols;
        for (int kk = 0; kk < p.k_stages && ok; ++kk) {
          if (!mbar_wait(&full[s], ph, abort, deadline)) {
            ok = false;
            break;
          }
          const uint32_t b_saddr = smem_u32(smem + s * C::kStageBytes + C::kAStage);
#pragma unroll
          for (int khalf = 0; khalf < 2; ++khalf) {
            // gate/up: uses (gate, khalf) and (up, khalf) sit at consecutive
            // ring positions; down: one use per K half.
            int slot2 = slot;
            uint32_t sph2 = sph;
            if (MODE == kGateUp) {
              slot2 = slot + 1;
              if (slot2 == NS) {
                slot2 = 0;
                sph2 ^= 1u;
              }
            }
            if (!mbar_wait(&afull[slot], sph, abort, deadline) ||
                (MODE == kGateUp && !mbar_wait(&afull[slot2], sph2, abort, deadline))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = tmem + slot * kSlotCols;
            const uint32_t a1 = tmem + slot2 * kSlotCols;
#pragma unroll
            for (int m = 0; m < 8; ++m) {
              const int kel = khalf * 128 + m * 16;
              const uint64_t bd = desc_sw128(b_saddr + (kel >> 6) * (BN * 128) + (kel & 63) * 2);
              const int step = (MODE == kGateUp ? 0 : khalf * 8) + m;  // step within K half pair
              const int part = step % C::kP;
              // a partial's first MMA of the unit overwrites it
              const uint32_t acc = (kk != 0 || khalf != 0 || step >= C::kP) ? 1u : 0u;
              const uint32_t accg = MODE == kGateUp ? ((kk != 0 || khalf != 0 || m >= C::kP) ? 1u : 0u) : acc;
              mma_f16_ts(d_tm + part * BN, a0 + m * 8, bd, C::kIdesc, accg);
              if (MODE == kGateUp)
                mma_f16_ts(d_tm + C::kOutCols + part * BN, a1 + m * 8, bd, C::kIdesc, accg);
            }
            mma_commit(&aempty[slot]);
            if (MODE == kGateUp) mma_commit(&aempty[slot2]);
            const int adv = MODE == kGateUp ? 2 : 1;
#pragma unroll
            for (int a = 0; a < adv; ++a) {
              if (++slot == NS) {
                slot = 0;
                sph ^= 1u;
              }
            }
          }
          if (!ok) break;
          mma_commit(&empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&dfull[d]);
      }
      // all MMAs issued by this thread complete before tensor memory is freed
      mma_commit(&done_bar);
      const uint64_t drain_deadline = now_ns() + kTimeoutNs;
      while (!mbar_try_wait(&done_bar, 0) && now_ns() < drain_deadline) {
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------- dequant into tensor memory ----------------
    const int wg = (warp - 4) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int s = 0;
    uint32_t ph = 0;
    int slot = wg;         // this warpgroup's position in the A ring
    uint32_t sph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      for (int kk = 0; kk < p.k_stages && ok; ++kk) {
        if (!warp_wait(&full[s], ph, abort, deadline)) {
          ok = false;
          break;
        }
        const uint8_t* st = smem + s * C::kStageBytes;
        const uint8_t* ss = st + C::kAStage + C::kBStage;
#pragma unroll
        for (int j = wg; j < C::kUsesPerStage; j += 2) {
          if (!warp_wait(&aempty[slot], sph ^ 1u, abort, deadline)) {
            ok = false;
            break;
          }
          // gate/up: warpgroup wg owns the gate (0) or up (1) rows and use j
          // selects the K half; down: warpgroup wg owns K half wg.
          const int arow = MODE == kGateUp ? wg * kM + row : row;
          const int khalf = MODE == kGateUp ? (j >> 1) : wg;
          const uint8_t* ap = st + arow * kRowBytes;
          uint4 qv[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int jj = khalf * 4 + c;
            qv[c] = *reinterpret_cast<const uint4*>(ap + ((jj ^ (arow & 7)) << 4));
          }
          const uint2 sc = *reinterpret_cast<const uint2*>(ss + arow * kRowScales + khalf * 8);
          uint32_t r[64];
          if (MODE == kGateUp) dequant_f16(qv, sc, r);
          else dequant_bf16(qv, sc, r);
          const uint32_t taddr = tmem + lane_base + slot * kSlotCols;
          tmem_st32(taddr, r);
          tmem_st32(taddr + 32, r + 32);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[slot]);
          // advance two ring positions: the other warpgroup takes the one between
#pragma unroll
          for (int step = 0; step < 2; ++step) {
            if (++slot == NS) {
              slot = 0;
              sph ^= 1u;
            }
          }
        }
        if (!ok) break;
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp >= 12) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint32_t ui = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++ui) {
      int e, nt, mt;
      decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
      const int d = ui % C::kDBufs;
      if (!warp_wait(&dfull[d], (ui / C::kDBufs) & 1u, abort, deadline)) break;
      tc_fence_after();
      const int valid = min(BN, p.counts[e] - nt * BN);
      const int slot0 = p.offsets[e] + nt * BN;
      const float gs = p.gscale[e];
      const uint32_t taddr = tmem + lane_base + C::kDCol0 + d * C::kDCols;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        {
          uint32_t t[16];
          tmem_ld16(taddr + c0, t);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(t[j]);
#pragma unroll
          for (int pp = 1; pp < C::kP; ++pp) {
            tmem_ld16(taddr + pp * BN + c0, t);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += __uint_as_float(t[j]);
          }
        }
        if (MODE == kGateUp) {
          float w[16];
          {
            uint32_t t[16];
            tmem_ld16(taddr + C::kOutCols + c0, t);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = __uint_as_float(t[j]);
#pragma unroll
            for (int pp = 1; pp < C::kP; ++pp) {
              tmem_ld16(taddr + C::kOutCols + pp * BN + c0, t);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) w[j] += __uint_as_float(t[j]);
            }
          }
          __nv_bfloat16* h = static_cast<__nv_bfloat16*>(p.out);
          const int f = mt * kM + r;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < valid) {
              const float sc = gs * p.xscale[slot0 + c0 + j];
              const float gv = v[j] * sc;
              const float uv = w[j] * sc;
              h[static_cast<int64_t>(slot0 + c0 + j) * p.out_ld + f] =
                  __float2bfloat16_rn(silu(gv) * uv);
            }
          }
        } else {
          float* y = static_cast<float*>(p.out);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < valid)
              y[static_cast<int64_t>(slot0 + c0 + j) * p.out_ld + mt * kM + r] = v[j] * gs;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (tid == 0 && abort_s) atomicOr(&p.status[1], 1u);
}

// Gather each sorted route's activation row as f16, scaled by a power of two
// so the row maximum lands in [2^14, 2^15): exact for bf16 and f16 inputs
// (bf16 keeps 8 significant bits, f16 11) down to 2^-24 of the row maximum.
__global__ void __launch_bounds__(256) gather_f16_kernel(
    const void* __restrict__ hidden, int act_dt, const int32_t* __restrict__ sorted,
    const int32_t* __restrict__ offsets, int E, int top_k, int K, __half* __restrict__ xperm,
    float* __restrict__ xscale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= offsets[E]) return;
  const int64_t token = sorted[warp] / top_k;
  float amax = 0.0f;
  if (act_dt == kBF16) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(hidden) +
                                                      token * K);
    for (int i = lane; i < K / 8; i += 32) {
      const uint4 v = src[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        amax = fmaxf(amax, fabsf(__uint_as_float(w[j] << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
      }
    }
  } else {
    for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(load_act(hidden, token * K + k, act_dt)));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  int ex = 0;
  if (amax > 0.0f && amax <= 3.0e38f) {
    frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
    ex -= 15;           // amax * 2^-ex in [2^14, 2^15)
  }
  const float down = ldexpf(1.0f, -ex);
  __half* dst = xperm + static_cast<int64_t>(warp) * K;
  if (act_dt == kBF16) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(hidden) +
                                                      token * K);
    for (int i = lane; i < K / 8; i += 32) {
      const uint4 v = src[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(w[j] << 16) * down,
                                             __uint_as_float(w[j] & 0xFFFF0000u) * down);
        o[j] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    for (int k = lane; k < K; k += 32)
      dst[k] = __float2half_rn(load_act(hidden, token * K + k, act_dt) * down);
  }
  if (lane == 0) xscale[warp] = ldexpf(1.0f, ex);
}

// ---- host side ----------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
               uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
               CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, int BN>
cudaError_t launch_one(const CUtensorMap& a, const CUtensorMap& s, const CUtensorMap& b,
                       const TcParams& p, int grid, cudaStream_t stream) {
  using C = Cfg<MODE, BN>;
  auto kern = moe_gemm_tc_kernel<MODE, BN>;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  static bool attr[64] = {};
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (err != cudaSuccess) return err;
    attr[dev] = true;
  }
  kern<<<grid, kThreads, C::kSmem, stream>>>(a, s, b, p);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_bn(int bn, const CUtensorMap& a, const CUtensorMap& s, const CUtensorMap& b,
                      const TcParams& p, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: return launch_one<MODE, 16>(a, s, b, p, grid, stream);
    case 32: return launch_one<MODE, 32>(a, s, b, p, grid, stream);
    case 64: return launch_one<MODE, 64>(a, s, b, p, grid, stream);
    case 128:
      if constexpr (MODE == kDown) return launch_one<kDown, 128>(a, s, b, p, grid, stream);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

bool tc_supported(int K, int I, int act_dt) {
  return act_dt != kF32 && K % kBK == 0 && I % kBK == 0 && get_encode() != nullptr;
}

int tc_token_tile(int64_t routes, int E, int mode) {
  const int64_t per = (routes + E - 1) / E;
  int bn = 16;
  while (bn < per && bn < (mode == kGateUp ? 64 : 128)) bn *= 2;
  return bn;
}

cudaError_t launch_moe_tc(const TcLaunch& a, cudaStream_t stream, const char** step) {
  const int64_t R = a.R;
  // 1. gather + f16 scaling of the sorted activation rows
  *step = "gather";
  {
    const int warps_per_block = 8;
    const int64_t blocks = (R + warps_per_block - 1) / warps_per_block;
    if (blocks > 0) {
      gather_f16_kernel<<<(unsigned)blocks, 32 * warps_per_block, 0, stream>>>(
          a.hidden, a.act_dt, a.sorted, a.offsets, a.E, a.top_k, a.K,
          static_cast<__half*>(a.xperm), a.xscale);
      cudaError_t err = cudaGetLastError();
      if (err != cudaSuccess) return err;
    }
  }
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 1);
  const int grid = sm_count();
  // 2. gate/up + SwiGLU
  *step = "gate/up tensor maps";
  {
    CUtensorMap ta, ts, tb;
    const int bn = tc_token_tile(R, a.E, kGateUp);
    if (!encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w13, a.K / 2, (uint64_t)a.E * 2 * a.I,
                   a.K / 2, kRowBytes, kM, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.s13, a.K / 16, (uint64_t)a.E * 2 * a.I,
                   a.K / 16, kRowScales, kM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.xperm, a.K, (uint64_t)(R > 0 ? R : 1),
                   (uint64_t)a.K * 2, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
    TcParams p{};
    p.counts = a.counts;
    p.offsets = a.offsets;
    p.gscale = a.g13;
    p.xscale = a.xscale;
    p.out = a.h;
    p.status = a.status;
    p.E = a.E;
    p.I = a.I;
    p.m_tiles = a.I / kM;
    p.k_stages = a.K / kBK;
    p.rows_per_expert = 2 * a.I;
    p.out_ld = a.I;
    *step = "gate/up";
    cudaError_t err = launch_bn<kGateUp>(bn, ta, ts, tb, p, grid, stream);
    if (err != cudaSuccess) return err;
  }
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 2);
  // 3. down projection
  *step = "down tensor maps";
  {
    CUtensorMap ta, ts, tb;
    const int bn = tc_token_tile(R, a.E, kDown);
    if (!encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w2, a.I / 2, (uint64_t)a.E * a.K, a.I / 2,
                   kRowBytes, kM, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.s2, a.I / 16, (uint64_t)a.E * a.K,
                   a.I / 16, kRowScales, kM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.h, a.I, (uint64_t)(R > 0 ? R : 1),
                   (uint64_t)a.I * 2, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
    TcParams p{};
    p.counts = a.counts;
    p.offsets = a.offsets;
    p.gscale = a.g2;
    p.xscale = nullptr;
    p.out = a.y;
    p.status = a.status;
    p.E = a.E;
    p.I = a.I;
    p.m_tiles = a.K / kM;
    p.k_stages = a.I / kBK;
    p.rows_per_expert = a.K;
    p.out_ld = a.K;
    *step = "down";
    cudaError_t err = launch_bn<kDown>(bn, ta, ts, tb, p, grid, stream);
    if (err != cudaSuccess) return err;
  }
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 3);
  return cudaSuccess;
}

}  // namespace sbb
