// Block-scaled tcgen05 path for the routed-expert NVFP4 MoE (sm_100a).
//
// The weights go to the tensor core as they are stored: packed e2m1 with one
// e4m3 scale per 16 elements, through tcgen05.mma kind::mxf4nvf4 block16
// (K = 64 per instruction, scales from tensor memory). Nothing dequantises a
// weight. A kind::f16 MMA that reads a 16-bit copy of the weights costs a
// fixed ~50 cycles per 128x16 weight tile whatever the token count, which at
// decode sizes is as slow as streaming the tile from HBM; the block-scaled
// instruction covers four times the weights per issue.
//
// The activations (bf16 hidden rows, then the fp32 SwiGLU rows) are split
// into NT NVFP4 terms by residual quantisation,
//   x = sum_t e2m1_t * e4m3_t * g_t  (+ residual),
// each 16-element block quantised with vLLM ref_nvfp4_quant semantics (the
// reference's fixture quantiser) under the per-row global g_t = g_0 / 4^t,
// g_0 = amax(x) / (448 * 6). A term shrinks a block's residual at least ~6x
// (about 11x typically), so the 4x step keeps every term's block scales in
// e4m3 range without a new row reduction per term, and each block runs its
// NT terms on its own. With NT = 4 the represented activations are within
// ~1e-4 (normwise) of the inputs, finer than the bf16 rounding of the inputs
// themselves. Two layouts of the terms:
//   rows  (decode-sized tiles): the terms of a row sit in consecutive rows of
//         the N operand, so one MMA covers all terms of BN/NT routed tokens
//         and the epilogue folds them: D[:, slot] = sum_t D[:, slot*NT + t] *
//         g_t. Few tokens per expert: N stays small and the MMA count low.
//   K     (prefill-sized tiles): term t of every slot sits in plane t
//         ([NT][R][K/2]); every term shares the row's global g_0 (the 4^-t
//         factor lives in the e4m3 block scales instead, same precision), so
//         x.W = sum_t x_t.W accumulates in one TMEM column per token: the MMA
//         runs over the NT planes as if they were a longer K. A weight tile
//         then serves NT times as many tokens per byte staged, which is what
//         bounds the prefill GEMMs (shared-memory fill rate from L2).
//
// A work unit is (expert, weight-row tile, token tile): 128 gate rows plus
// the matching 128 up rows (gate/up), or 256 consecutive w2 rows (down),
// against BN term rows of that expert's routed tokens. A persistent grid of
// one CTA per SM walks the units; within a CTA the warps specialise:
//   warp 0       TMA: packed weights (128-byte swizzle), their linear scale
//                rows, the packed term rows and their scale rows.
//   warp 1       TMEM allocation; one thread issues the MMAs.
//   warps 2-3    down tiles of prefill-sized calls only: the second 128-row
//                weight block of each stage by cp.async, a second queue of
//                requests beside the TMA (decode calls, with inline plans:
//                the route histogram in the prologue).
//   warps 4-7    scale warps: write the stage's e4m3 scales into tensor
//                memory with tcgen05.st in the layout the block-scaled MMA
//                reads: for a 128-row operand block and a 64-wide K group the
//                4 scales of row r0 + 32*r1 sit in column c + r1 of lane r0
//                of every 32-lane quarter. Writing them from registers keeps
//                the tensor core's queue for MMAs only (a tcgen05.cp costs as
//                much as an MMA there, and mixing the two serialises).
//   warps 8-15   epilogue, two teams of four warps on alternate 16-column
//                chunks: fold terms, global scale, SwiGLU (gate/up) or the
//                fp32 route output (down).
// Every wait is bounded (the kernel raises status[1], drains and returns).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "tc_ptx.cuh"

namespace sbb {

namespace {

using namespace ptx;

constexpr int kBK = 256;              // K elements per pipeline stage
// Mean routes per expert from which the activation terms go along K.
constexpr double kKtMinTokens = 96.0;
// Terms of the K layout. Three residual NVFP4 terms represent a bf16 row to
// ~8e-4 (normwise; four: ~8e-5), finer than the bf16 rounding of the row
// itself (~1e-3). At prefill sizes the GEMMs are bound by how many staged
// bytes each SM keeps in flight, and the term planes are most of them: three
// planes stage 90 KB per 128-token gate/up step instead of 108 KB and issue a
// quarter fewer MMAs.
constexpr int kKtTerms = 3;
// Threads (warps 2-3) that copy the second weight block of every stage with
// cp.async when the weights are L2-resident (prefill-sized calls): the
// load/store path adds a second queue of requests in flight to the TMA's.
constexpr int kLsuThreads = 64;
constexpr int kRowBytes = kBK / 2;    // packed bytes per row per stage (128)
constexpr int kRowScales = kBK / 16;  // scale bytes per row per stage (16)
constexpr int kM = 128;
constexpr int kThreads = 512;
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // default wait limit; drains always get this

// Limit of the pipeline waits of the grouped GEMMs (sbb200_set_kernel_wait_ns).
std::atomic<uint64_t> g_wait_ns{kTimeoutNs};

// Error bits of every GEMM launch on this device since the host last read
// them (sbb200_device_errors): unlike the per-call word in the workspace,
// which each call clears, this one keeps a failure of any earlier call, so a
// run of graph replays can be checked once at its end. Zero at load.
__device__ uint32_t g_sticky_errors = 0;

enum : int { kGateUp = 0, kDown = 1 };

struct BsParams {
  const int32_t* counts;
  const int32_t* offsets;
  const float* gscale;  // per-expert weight global (g13 or g2)
  const float* bg;      // per (slot, term) activation global
  float* out;           // gate/up: fp32 h [R, I]; down: fp32 y [R, K]
  uint32_t* status;
  int E;
  int I;
  int m_tiles;          // I/128 (gate/up) or K/256 (down)
  int a_stride;         // row offset of the second 128-row block: I (up rows) or 128
  int k_stages;         // reduction / 256
  int rows_per_expert;  // 2I or K
  int out_ld;           // I or K
  int stream_weights;   // 1: each weight tile is read by about one token tile
                        // (decode): weights evict_first, term rows evict_last;
                        // 0: tiles are shared by several token tiles in
                        // flight (prefill): both evict_normal
  uint64_t wait_ns;     // limit of every pipeline wait, counted from the
                        // moment the previous kernel's results are visible
  // down, expert parallel: rows go to their source ranks (PushRows), found
  // through the route id of each slot
  const int32_t* sorted;
  float* const* push_base;
  int64_t push_rows;
  int top_k;
  // K-layout tiles: the term scales come in as contiguous runs of bsf
  // ([plane][k stage][slot][16], `plane` rows each)
  const uint8_t* bsf;
  int64_t plane;
  // calls whose route plan is computed inside the activation split (at most
  // kInlinePlanRoutes routes, ids given): the call's route ids. The kernel
  // then derives the plan's counts and first slots from them itself and
  // streams its first stages of weights before the previous kernel has
  // finished (only the term rows wait for it).
  const int32_t* early_ids;
  int early_routes;
  // the weight plane (w13 or w2) and its row length in bytes. With lsu_half
  // the second 128-row weight block of each stage is copied by warps 2-3
  // with cp.async (the load/store path), the rest by TMA: for down tiles whose
  // weights are shared by several token tiles (L2-resident), where one
  // SM's TMA requests in flight bound the fill rate; streamed weights (decode)
  // come faster through TMA alone.
  const uint8_t* wa;
  int64_t wa_ld;
  int lsu_half;
};

// BNR: the MMA's N. KT = false: N = BNR term rows (BNR / NT tokens, terms
// interleaved); KT = true: N = BNR tokens, their NT term planes staged one
// after the other and run as NT K-slices into the same accumulator.
template <int MODE, int BNR, int NT, bool KT = false>
struct BsCfg {
  // two 128-row weight blocks per unit: gate and up rows (gate/up) or 256
  // consecutive rows of w2 (down), each into its own accumulator
  static constexpr int kNA = 2;
  static constexpr int kTok = KT ? BNR : BNR / NT;         // routed tokens per tile
  static constexpr int kBSets = KT ? NT : 1;               // B operands per K group
  static constexpr int kA = kNA * kM * kRowBytes;          // packed weights
  static constexpr int kB = kBSets * BNR * kRowBytes;      // packed term rows
  static constexpr int kSA = kNA * kM * kRowScales;        // linear weight scales
  static constexpr int kSB = kBSets * BNR * kRowScales;    // linear term scales
  static constexpr int kRaw = kA + kB + kSA + kSB;
  static constexpr int kStageBytes = (kRaw + 1023) / 1024 * 1024;
  static constexpr int kStagesRaw = (224 * 1024 - 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  static constexpr int kOffB = kA;
  static constexpr int kOffSA = kA + kB;
  static constexpr int kOffSB = kOffSA + kSA;
  // tensor memory: accumulators, then the scale buffers. Row n of an operand
  // keeps the 4 scales of a 64-wide K group in column n / 32 of that group's
  // columns, lane n % 32 of every 32-lane quarter: a 128-row A block takes 4
  // columns per K group, B takes 4 (up to 128 rows) or 8 (up to 256), so
  // every scale address handed to the MMA is 4-column aligned; B fills the
  // first ceil(rows / 32) of its columns and zeroes the rest. With KT each
  // term plane t has its own B scale columns: group kg of plane t at
  // (t * 4 + kg) * kBC.
  static constexpr int kDCols = kNA * BNR;
  static constexpr int kBQ = (BNR + 31) / 32;        // B row quarters in use
  static constexpr int kBC = BNR > 128 ? 8 : 4;      // B scale columns per K group
  // per buffer, a multiple of 16 so every tcgen05.st (x4/x8/x16) starts on a
  // column aligned to its width
  static constexpr int kSfCols = kNA * 16 + kBSets * 4 * kBC;
  static constexpr int kDBufs = 2 * kDCols + 2 * kSfCols <= kTmemCols ? 2 : 1;
  static constexpr int kSfCol0 = kDBufs * kDCols;
  // scale-factor ring: as many buffers as tensor memory leaves room for, up
  // to 4, so the scale warps can run that many stages ahead of the MMAs
  static constexpr int kSfFit = (kTmemCols - kSfCol0) / kSfCols;
  static constexpr int kSfBufs = kSfFit > 4 ? 4 : kSfFit;
  static constexpr uint32_t kIdesc =
      (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BNR >> 3) << 17) | ((kM >> 4) << 24);
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert(kSfCol0 % 16 == 0 && kSfCols % 16 == 0, "tensor-memory store alignment");
  static_assert(kSfBufs >= 2 && kSfCol0 + kSfBufs * kSfCols <= kTmemCols, "tensor memory");
  static_assert(BNR % 16 == 0 && BNR >= 16 && BNR <= 256 && (KT || BNR % NT == 0), "tile");
  static_assert(!KT || (BNR * kRowBytes) % 1024 == 0, "term planes keep the 1024-byte swizzle atom");
};

__device__ __forceinline__ void decode_unit(int u, int m_tiles, const int* prefix, int E, int& e,
                                            int& nt, int& mt) {
  const int t = u / m_tiles;
  mt = u - t * m_tiles;
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  e = lo;
  nt = t - prefix[e];
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  for (uint32_t i = 0;; ++i) {
    const bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    if ((i & 15) == 0) {
      int stop = 0;
      if (lane == 0) {
        stop = *abort || now_ns() > deadline;
        if (stop) *abort = 1;
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}


__device__ __forceinline__ void mma_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

template <int MODE, int BNR, int NT, bool KT>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_bs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmSA,
                       const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmSB,
                       const BsParams p) {
  using C = BsCfg<MODE, BNR, NT, KT>;
  constexpr int S = C::kStages;
  constexpr int NB = C::kDBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr int NSF = C::kSfBufs;
  __shared__ __align__(8) uint64_t full[S], empty[S], sfready[NSF], dfull[NB], dempty[NB],
      sffree[NSF], done_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ int prefix[kMaxExperts + 1];
  // per-expert routed count, first slot and weight global, staged once so
  // the producer and the epilogue read shared memory at every unit start
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_off[kMaxExperts];
  __shared__ float s_gs[kMaxExperts];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  volatile int* abort = &abort_s;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1 + (p.lsu_half ? kLsuThreads : 0));  // TMA + the cp.async threads
      mbar_init(&empty[i], 1 + 4);  // MMA commit + the four scale warps
    }
    for (int i = 0; i < NSF; ++i) {
      mbar_init(&sfready[i], 4);
      mbar_init(&sffree[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 8);  // both epilogue teams
    }
    mbar_init(&done_bar, 1);
    abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmSA);
    prefetch_tensormap(&tmB);
    prefetch_tensormap(&tmSB);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  // everything above is local to the CTA. Without early_ids the kernel now
  // waits for the previous kernel (its results are read from here on); with
  // them it reads only the call's inputs until each role's own wait below.
  const bool early = p.early_ids != nullptr;
  if (!early) {
    pdl_wait();
    pdl_trigger();
  }
  if (warp == 2 || warp == 3) {
    const int t64 = tid - 64;
    if (early) {
      // the route plan's counts (ids outside [0, E) dropped) and first slots
      // (exclusive scan), as the activation split computes them
      for (int e = t64; e < p.E; e += 64) {
        s_cnt[e] = 0;
        s_gs[e] = p.gscale[e];
      }
      asm volatile("bar.sync 2, 64;" ::: "memory");
      for (int r = t64; r < p.early_routes; r += 64) {
        const int32_t e = p.early_ids[r];
        if (e >= 0 && e < p.E) atomicAdd(&s_cnt[e], 1);
      }
      asm volatile("bar.sync 2, 64;" ::: "memory");
      if (warp == 2) {
        int carry = 0;
        for (int e0 = 0; e0 < p.E; e0 += 32) {
          const int e = e0 + lane;
          const int v = e < p.E ? s_cnt[e] : 0;
          int incl = v;
#pragma unroll
          for (int d = 1; d < 32; d <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += n;
          }
          if (e < p.E) s_off[e] = carry + incl - v;
          carry += __shfl_sync(0xffffffffu, incl, 31);
        }
      }
    } else {
      // every expert's count, first slot and global in one batch of loads
      // (kMaxExperts / 64 per thread)
      for (int e = t64; e < p.E; e += 64) {
        s_cnt[e] = p.counts[e];
        s_off[e] = p.offsets[e];
        s_gs[e] = p.gscale[e];
      }
    }
    asm volatile("bar.sync 2, 64;" ::: "memory");
    // warp 2 scans the tile counts
    if (warp == 2) {
      int carry = 0;
      for (int e0 = 0; e0 < p.E; e0 += 32) {
        const int e = e0 + lane;
        int v = e < p.E ? (s_cnt[e] + C::kTok - 1) / C::kTok : 0;
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
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  const int total_units = prefix[p.E] * p.m_tiles;
  // early: every role but the producer now waits for the previous kernel
  // (the producer first issues its first stages of weights)
  const bool producer = (warp == 0 && lane == 0) || (p.lsu_half && (warp == 2 || warp == 3));
  if (early && !producer) {
    pdl_wait();
    pdl_trigger();
  }
  // the wait limit runs from the dependency wait, so a long predecessor does
  // not eat into it (the producer restarts it after its own wait)
  uint64_t deadline = now_ns() + p.wait_ns;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = p.stream_weights ? policy_evict_first() : policy_evict_normal();
      const uint64_t pol_x = p.stream_weights ? policy_evict_last() : policy_evict_normal();
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[S];
      bool issued[S];
#pragma unroll
      for (int i = 0; i < S; ++i) issued[i] = false;
      bool ok = true;
      // the weight half of a stage: packed weight rows and their scales
      auto load_weights = [&](int st_i, int e, int mt, int kk) {
        uint8_t* st = smem + st_i * C::kStageBytes;
        const int r0 = e * p.rows_per_expert + mt * (MODE == kGateUp ? kM : 2 * kM);
#pragma unroll
        for (int a = 0; a < C::kNA; ++a) {
          if (a == 0 || !p.lsu_half)  // with lsu_half warps 2-3 bring the second block
            tma_load_2d_hint(st + a * kM * kRowBytes, &tmA, &full[st_i], kk * kRowBytes,
                             r0 + a * p.a_stride, pol_w);
          tma_load_2d_hint(st + C::kOffSA + a * kM * kRowScales, &tmSA, &full[st_i],
                           kk * kRowScales, r0 + a * p.a_stride, pol_w);
        }
      };
      // the term half of a stage: the activation (or SwiGLU) term rows and
      // their scales, which the previous kernel wrote
      auto load_terms = [&](int st_i, int row_b, int kk) {
        uint8_t* st = smem + st_i * C::kStageBytes;
        if (KT) {
          // all NT planes of the tile's slots in one box: [plane][slot][bytes];
          // their scales are one contiguous run per plane, moved by a plain
          // bulk copy rather than a box of 16-byte rows
          tma_load_3d_hint(st + C::kOffB, &tmB, &full[st_i], kk * kRowBytes, row_b, 0, pol_x);
#pragma unroll
          for (int t = 0; t < NT; ++t)
            bulk_load_hint(st + C::kOffSB + t * BNR * kRowScales,
                           p.bsf + ((static_cast<int64_t>(t) * p.k_stages + kk) * p.plane +
                                    row_b) * kRowScales,
                           BNR * kRowScales, &full[st_i], pol_x);
        } else {
          tma_load_2d_hint(st + C::kOffB, &tmB, &full[st_i], kk * kRowBytes, row_b, pol_x);
          tma_load_2d_hint(st + C::kOffSB, &tmSB, &full[st_i], kk * kRowScales, row_b, pol_x);
        }
      };
      // first term row (rows layout) or first slot (KT: the planes' y) of a unit
      auto term_row = [&](int e, int nt) { return (s_off[e] + nt * C::kTok) * (KT ? 1 : NT); };
      int u0 = blockIdx.x, kk0 = 0;  // where the main loop starts
      if (early) {
        // the first stages' weights before the dependency wait (the ring is
        // still empty, so nothing to wait for), their term rows after it
        int n_early = 0, eu[S], ekk[S];
        while (n_early < S && u0 < total_units) {
          int e, nt, mt;
          decode_unit(u0, p.m_tiles, prefix, p.E, e, nt, mt);
          mbar_expect_tx(&full[n_early], C::kA - (p.lsu_half ? kM * kRowBytes : 0) + C::kB + C::kSA + C::kSB);
          load_weights(n_early, e, mt, kk0);
          issued[n_early] = true;
          issued_phase[n_early] = 0;
          eu[n_early] = u0;
          ekk[n_early] = kk0;
          ++n_early;
          if (++kk0 == p.k_stages) {
            kk0 = 0;
            u0 += gridDim.x;
          }
        }
        pdl_wait();
        pdl_trigger();
        deadline = now_ns() + p.wait_ns;
        for (int i = 0; i < n_early; ++i) {
          int e, nt, mt;
          decode_unit(eu[i], p.m_tiles, prefix, p.E, e, nt, mt);
          load_terms(i, term_row(e, nt), ekk[i]);
        }
        s = n_early % S;
        ph = n_early == S ? 1u : 0u;
      }
      for (int u = u0; u < total_units && ok; u += gridDim.x) {
        int e, nt, mt;
        decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
        const int row_b = term_row(e, nt);
        for (int kk = (u == u0 ? kk0 : 0); kk < p.k_stages; ++kk) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort, deadline)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], C::kA - (p.lsu_half ? kM * kRowBytes : 0) + C::kB + C::kSA + C::kSB);
          load_weights(s, e, mt, kk);
          load_terms(s, row_b, kk);
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      const uint64_t drain_deadline = now_ns() + kTimeoutNs;
      for (int i = 0; i < S; ++i) {
        if (!issued[i]) continue;
        while (!mbar_try_wait(&full[i], issued_phase[i]) && now_ns() < drain_deadline) {
        }
      }
    }
  } else if (p.lsu_half && (warp == 2 || warp == 3)) {
    // ---------------- second weight block by cp.async ----------------
    const int lt = tid - 64;
    auto issue = [&](int st_i, int e, int mt, int kk) {
      uint8_t* dst = smem + st_i * C::kStageBytes + kM * kRowBytes;
      const int64_t r0 = static_cast<int64_t>(e) * p.rows_per_expert +
                         mt * (MODE == kGateUp ? kM : 2 * kM) + p.a_stride;
      const uint8_t* src = p.wa + r0 * p.wa_ld + kk * kRowBytes;
      // 128 rows x 8 chunks of 16 bytes, in the 128-byte swizzle the MMA's
      // descriptor expects (chunk c of row r at c ^ (r % 8))
#pragma unroll 4
      for (int i = lt; i < kM * 8; i += kLsuThreads) {
        const int r = i >> 3, c = i & 7;
        cp_async16(dst + r * kRowBytes + ((c ^ (r & 7)) << 4), src + r * p.wa_ld + c * 16);
      }
      cp_async_arrive(&full[st_i]);
    };
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    int u0 = blockIdx.x, kk0 = 0;
    if (early) {
      int n_early = 0;
      while (n_early < S && u0 < total_units) {
        int e, nt, mt;
        decode_unit(u0, p.m_tiles, prefix, p.E, e, nt, mt);
        issue(n_early, e, mt, kk0);
        ++n_early;
        if (++kk0 == p.k_stages) {
          kk0 = 0;
          u0 += gridDim.x;
        }
      }
      pdl_wait();
      pdl_trigger();
      deadline = now_ns() + p.wait_ns;
      s = n_early % S;
      ph = n_early == S ? 1u : 0u;
    }
    for (int u = u0; u < total_units && ok; u += gridDim.x) {
      int e, nt, mt;
      decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
      for (int kk = (u == u0 ? kk0 : 0); kk < p.k_stages; ++kk) {
        if (!warp_wait(&empty[s], ph ^ 1u, abort, deadline)) {
          ok = false;
          break;
        }
        issue(s, e, mt, kk);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    cp_async_wait_all();
  } else if (warp == 1) {
    // ---------------- scale copies + MMA issuer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t it = 0;  // stage sequence number (scale buffer = it % NSF)
      uint32_t ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++ui) {
        const int d = ui % NB;
        // the MMA's N covers the tile's routed tokens (rounded up to 16 rows),
        // so an expert's last, partly filled tile costs only what it holds
        int e, nt, mt;
        decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
        const int valid = min(C::kTok, s_cnt[e] - nt * C::kTok);
        const int n_rows = KT ? valid : valid * NT;
        const int n_mma = min(BNR, max(16, (n_rows + 15) & ~15));
        const uint32_t idesc = (C::kIdesc & ~(0x3Fu << 17)) | (static_cast<uint32_t>(n_mma >> 3) << 17);
        if (!mbar_wait(&dempty[d], ((ui / NB) & 1u) ^ 1u, abort, deadline)) break;
        tc_fence_after();
        const uint32_t d_tm = tmem + d * C::kDCols;
        for (int kk = 0; kk < p.k_stages; ++kk) {
          const int sb = it % NSF;
          if (!mbar_wait(&full[s], ph, abort, deadline) ||
              !mbar_wait(&sfready[sb], (it / NSF) & 1u, abort, deadline)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + s * C::kStageBytes;
          const uint32_t a_sa = smem_u32(st);
          const uint32_t b_sa = smem_u32(st + C::kOffB);
          const uint32_t sf0 = tmem + C::kSfCol0 + sb * C::kSfCols;
#pragma unroll
          for (int kg = 0; kg < 4; ++kg) {
#pragma unroll
            for (int t = 0; t < C::kBSets; ++t) {
              const uint64_t bd = desc_sw128(b_sa + t * BNR * kRowBytes + kg * 32);
              const uint32_t acc = (kk | kg | t) != 0;
#pragma unroll
              for (int a = 0; a < C::kNA; ++a) {
                const uint64_t ad = desc_sw128(a_sa + a * kM * kRowBytes + kg * 32);
                mma_bs(d_tm + a * BNR, ad, bd, idesc, sf0 + a * 16 + kg * 4,
                       sf0 + C::kNA * 16 + (t * 4 + kg) * C::kBC, acc);
              }
            }
          }
          mma_commit(&empty[s]);
          mma_commit(&sffree[sb]);
          ++it;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&dfull[d]);
      }
      mma_commit(&done_bar);
      const uint64_t drain_deadline = now_ns() + kTimeoutNs;
      while (!mbar_try_wait(&done_bar, 0) && now_ns() < drain_deadline) {
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- scales into tensor memory ----------------
    const int q = warp & 3;  // this warp's 32-lane quarter of tensor memory
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int s = 0;
    uint32_t ph = 0;
    uint32_t it = 0;  // stage sequence number (scale buffer = it % NSF)
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      for (int kk = 0; kk < p.k_stages; ++kk) {
        const int sb = it % NSF;
        // the buffer's previous MMAs (NSF stages ago) are complete
        if (!warp_wait(&full[s], ph, abort, deadline) ||
            !warp_wait(&sffree[sb], ((it / NSF) & 1u) ^ 1u, abort, deadline)) {
          ok = false;
          break;
        }
        const uint8_t* st = smem + s * C::kStageBytes;
        const uint32_t sf0 = tmem + lane_base + C::kSfCol0 + sb * C::kSfCols;
        // column kg*4 + r1 of lane r0: word kg (4 scales) of row r0 + 32*r1
        uint32_t ra[16];
#pragma unroll
        for (int a = 0; a < C::kNA; ++a) {
#pragma unroll
          for (int r1 = 0; r1 < 4; ++r1) {
            const uint4 v = *reinterpret_cast<const uint4*>(
                st + C::kOffSA + (a * kM + r1 * 32 + lane) * kRowScales);
            ra[0 * 4 + r1] = v.x;
            ra[1 * 4 + r1] = v.y;
            ra[2 * 4 + r1] = v.z;
            ra[3 * 4 + r1] = v.w;
          }
          tmem_st16(sf0 + a * 16, ra);
        }
        constexpr int BC = C::kBC;
#pragma unroll 1
        for (int t = 0; t < C::kBSets; ++t) {
          uint32_t rb[4 * BC];
#pragma unroll
          for (int r1 = 0; r1 < BC; ++r1) {
            const int n = r1 * 32 + lane;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r1 < C::kBQ && n < BNR)
              v = *reinterpret_cast<const uint4*>(st + C::kOffSB + (t * BNR + n) * kRowScales);
            rb[0 * BC + r1] = v.x;
            rb[1 * BC + r1] = v.y;
            rb[2 * BC + r1] = v.z;
            rb[3 * BC + r1] = v.w;
          }
#pragma unroll
          for (int c = 0; c < 4 * BC; c += 16)
            tmem_st16(sf0 + C::kNA * 16 + t * 4 * BC + c, rb + c);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sfready[sb]);
          mbar_arrive(&empty[s]);
        }
        ++it;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp >= 8) {
    // ---------------- epilogue: two teams of four warps ----------------
    // warps 8-11 and 12-15 each cover the four 32-lane quarters and take
    // alternate 16-column chunks, so the accumulator drains twice as fast
    const int q = warp & 3;
    const int team = (warp >> 2) & 1;
    const int r = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint32_t ui = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++ui) {
      int e, nt, mt;
      decode_unit(u, p.m_tiles, prefix, p.E, e, nt, mt);
      const int d = ui % NB;
      if (!warp_wait(&dfull[d], (ui / NB) & 1u, abort, deadline)) break;
      tc_fence_after();
      const int valid = min(C::kTok, s_cnt[e] - nt * C::kTok);
      const int slot0 = s_off[e] + nt * C::kTok;
      const float gs = s_gs[e];
      const uint32_t taddr = tmem + lane_base + d * C::kDCols;
      // columns past the tile's last token were not written by the MMA
      const int n_cols = KT ? valid : valid * NT;
#pragma unroll 1
      for (int c0 = team * 16; c0 < n_cols; c0 += 32) {
        uint32_t t0[16], t1[16];
        tmem_ld16(taddr + c0, t0);
        tmem_ld16(taddr + BNR + c0, t1);
        constexpr int kTokPerChunk = KT ? 16 : 16 / NT;
        // expert parallel: lane l finds the source row of the chunk's token l
        // once (route r = v * top_k + k of virtual token v = src * rows + t
        // goes to row t * top_k + k of the source's buffer); the other lanes
        // take it by shuffle
        float* push_row = nullptr;
        if (MODE == kDown && p.push_base) {
          const int jl = (KT ? c0 : c0 / NT) + lane;
          if (lane < kTokPerChunk && jl < valid) {
            const int32_t rv = p.sorted[slot0 + jl];
            const int32_t v = rv / p.top_k;
            const int32_t src = v / static_cast<int32_t>(p.push_rows);
            push_row = p.push_base[src] +
                       (static_cast<int64_t>(v - src * static_cast<int32_t>(p.push_rows)) *
                            p.top_k + (rv - v * p.top_k)) * p.out_ld;
          }
        }
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < kTokPerChunk; ++jj) {
          const int j = KT ? c0 + jj : c0 / NT + jj;  // token within the tile
          if (j < valid) {
            const int slot = slot0 + j;
            float v0 = 0.0f, v1 = 0.0f;
            if (KT) {
              // the MMA summed the terms; they share the slot's global
              const float g = p.bg[slot];
              v0 = __uint_as_float(t0[jj]) * g;
              v1 = __uint_as_float(t1[jj]) * g;
            } else {
#pragma unroll
              for (int tt = 0; tt < NT; ++tt) {
                const float g = p.bg[static_cast<int64_t>(slot) * NT + tt];
                v0 = fmaf(__uint_as_float(t0[jj * NT + tt]), g, v0);
                v1 = fmaf(__uint_as_float(t1[jj * NT + tt]), g, v1);
              }
            }
            float* orow = p.out + static_cast<int64_t>(slot) * p.out_ld;
            if (MODE == kDown && p.push_base) {
              orow = reinterpret_cast<float*>(__shfl_sync(
                  0xffffffffu, reinterpret_cast<unsigned long long>(push_row), jj));
            }
            if (MODE == kGateUp) {
              const float gv = v0 * gs, uv = v1 * gs;
              orow[mt * kM + r] = silu(gv) * uv;
            } else {
              orow[mt * 2 * kM + r] = v0 * gs;
              orow[mt * 2 * kM + kM + r] = v1 * gs;
            }
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
  if (tid == 0 && abort_s) {
    atomicOr(&p.status[1], 1u);
    atomicOr(&g_sticky_errors, 1u);
  }
}

// ---- activation splitter ----------------------------------------------------

// Two fp32 -> one byte of e2m1 (lo -> low nibble), round to nearest even,
// saturating: cvt.rn.satfinite.e2m1x2.f32 places its first source operand in
// the upper nibble.
__device__ __forceinline__ uint32_t e2m1x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("{\n .reg .b8 b;\n cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n cvt.u32.u8 %0, b;\n}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float e4m3_to_f32_hw(uint32_t byte) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(static_cast<uint16_t>(byte & 0xFFu)));
  return __low2float(*reinterpret_cast<const __half2*>(&h));
}

__device__ __forceinline__ float2 e2m1x2_to_float2(uint32_t byte) {
  uint32_t h;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}" : "=r"(h) : "r"(byte));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}


// Splits rows into NT NVFP4 terms. One CTA per source row, one 16-element
// block per thread (blockDim: K / 16 rounded up to whole warps, at least
// kSplitThreads), so block maxima need no shuffles, the row maximum is one
// CTA reduction of values already in registers, every element is read once
// and a thread's packed block is one 8-byte store. Without slot_of, row i is
// written to output rows i*NT + t; with slot_of (token mode) source row i is
// token i and its terms go to every route slot the token feeds
// (slot_of[i*top_k + k], -1 skipped), so a token is split once however many
// experts it visits, and a token with no slot is not read at all. In token
// mode with an InlinePlan the slots are computed here instead of read.
// Outputs: packed e2m1 [row*NT + t, K/2], e4m3 scales [row*NT + t, K/16] and
// the dequant global g [row*NT + t].
constexpr int kSplitThreads = 64;

// CG: read through L2 only. Rows on another GPU are rewritten every step by
// their owner; an L1 line left from an earlier step on this SM would be
// stale, so they are never read through L1.
template <bool CG = false>
__device__ __forceinline__ void load8(const void* src, int src_dt, int64_t at, float* v) {
  if (src_dt == kF32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(src) + at);
    const float4 a = CG ? __ldcg(p) : p[0];
    const float4 b = CG ? __ldcg(p + 1) : p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + at);
    const uint4 w = CG ? __ldcg(p) : p[0];
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (src_dt == kBF16) {
        v[2 * i] = __uint_as_float(u[i] << 16);
        v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  }
}

// One 16-element block to one NVFP4 term under quantisation global G (g =
// 1/G): scale = min(G * bmax / 6, 448) to e4m3, elements to the nearest e2m1
// of x / (e4m3 * g) (vLLM ref_nvfp4_quant). With RESID the block is left
// holding what the term does not represent.
template <bool RESID>
__device__ __forceinline__ void quant_block(float* v, float G, float g, uint32_t* w,
                                            uint8_t* scale_byte) {
  float bmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  const float scale = fminf(__fmul_rn(G, __fmul_rn(bmax, 1.0f / 6.0f)), 448.0f);
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(scale, __NV_SATFINITE, __NV_E4M3);
  const float sg = __fmul_rn(e4m3_to_f32_hw(s8), g);  // one e2m1 step of this block
  const float inv = sg == 0.0f ? 0.0f : __frcp_rn(sg);
  w[0] = w[1] = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    // nearest e2m1 (ties to even, saturating at 6) of both elements
    const uint32_t pair = e2m1x2_from_f32(__fmul_rn(v[2 * j], inv), __fmul_rn(v[2 * j + 1], inv));
    if (RESID) {
      // the MMA sees e2m1 * e4m3 * g; the next term quantises what is left
      const float2 dq = e2m1x2_to_float2(pair);
      v[2 * j] -= __fmul_rn(dq.x, sg);
      v[2 * j + 1] -= __fmul_rn(dq.y, sg);
    }
    w[j >> 2] |= pair << (8 * (j & 3));
  }
  *scale_byte = static_cast<uint8_t>(s8);
}

// The dynamic-global split of one row held in registers, one 16-element
// block per thread (v; active: the block lies inside the row): the row
// maximum by a CTA reduction, then NT residual terms written to every
// destination slot dst[d] (d < ndst, -1 skipped), or to `row` alone when dst
// is null. Rows layout (plane = 0): term t of slot d is row d * NT + t,
// quantised under G0 * 4^t, with global gout[d * NT + t]. K layout (plane =
// R, the plane height): term t of slot d is row t * plane + d, every term
// under G0 (the e4m3 block scales carry the shrinking residual), one global
// gout[d]. Every thread of the CTA calls it; s_max holds 32 floats.
__device__ __forceinline__ void split_row_terms(float* v, bool active, int NT, int K,
                                                const int32_t* dst, int ndst, int64_t row,
                                                uint8_t* q, uint8_t* sf, float* gout,
                                                float* s_max, int64_t plane = 0) {
  const int tid = threadIdx.x;
  const int nwarps = blockDim.x >> 5;
  const int blk = tid;
  float amax = 0.0f;
  if (active) {
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  if ((tid & 31) == 0) s_max[tid >> 5] = amax;
  __syncthreads();
  amax = s_max[0];
  for (int w = 1; w < nwarps; ++w) amax = fmaxf(amax, s_max[w]);
  const float G0 = amax > 0.0f ? __fdiv_rn(2688.0f, amax) : 1.0f;
  const float g0 = __fdiv_rn(1.0f, G0);
  if (tid < ndst) {
    const int64_t d = dst ? static_cast<int64_t>(dst[tid]) : row;
    if (d >= 0) {
      if (plane) gout[d] = g0;
      else
        for (int t = 0; t < NT; ++t) gout[d * NT + t] = ldexpf(g0, -2 * t);
    }
  }
  if (!active) return;
  float G = G0, g = g0;
  for (int t = 0; t < NT; ++t) {
    uint32_t w[2];
    uint8_t s8;
    quant_block<true>(v, G, g, w, &s8);
    for (int i = 0; i < ndst; ++i) {
      const int64_t d = dst ? static_cast<int64_t>(dst[i]) : row;
      if (d < 0) continue;
      const int64_t orow = plane ? t * plane + d : d * NT + t;
      *reinterpret_cast<uint2*>(q + orow * (K / 2) + blk * 8) = make_uint2(w[0], w[1]);
      // K layout: scales stage-major, [plane][K / 256][slot][16], so a tile's
      // scales for one stage are one contiguous run
      const int64_t at = plane ? ((static_cast<int64_t>(t) * (K / 256) + blk / 16) * plane + d) *
                                         16 + (blk & 15)
                               : orow * (K / 16) + blk;
      sf[at] = s8;
    }
    if (!plane) {
      G = __fmul_rn(G, 4.0f);
      g = __fmul_rn(g, 0.25f);
    }
  }
}

// Route plan of a small call (R = gridDim.x * top_k <= kInlinePlanRoutes
// routes, blockDim >= kSplitThreads) computed inside the token-mode split, so
// no separate plan kernel runs ahead of it. Every CTA histograms all route
// ids in shared memory and scans the counts into expert offsets; the slot of
// its token's route r = row * top_k + i with expert e is then offsets[e] +
// #{r' < r : ids[r'] == e}, the stable (token, k) order of the separate plan
// (route_scatter_kernel). Each CTA writes its token's slot_of and sorted
// entries, CTA 0 also counts, offsets and the number of ids outside [0, E)
// other than -1.
struct InlinePlan {
  const int32_t* ids;  // nullptr: the route plan ran and the split reads its slot_of
  int E;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* slot_of;
  uint32_t* status;
};
constexpr int kInlinePer = kInlinePlanRoutes / kSplitThreads;  // route ids per thread

// s_off: kMaxExperts + 1 entries; s_rank, s_exp, s_dst: top_k entries.
// id_of(r) is the expert id of route r (r < R = gridDim.x * top_k); ids
// outside [0, E) are dropped, and counted in *status unless they are -1.
// Ends with every s_dst entry written and visible to the CTA.
template <class IdOf>
__device__ __forceinline__ void plan_route_slots(IdOf id_of, int E, int64_t row, int top_k,
                                                 int32_t* counts, int32_t* offsets,
                                                 int32_t* sorted, int32_t* slot_of,
                                                 uint32_t* status, int32_t* s_off,
                                                 int32_t* s_rank, int32_t* s_exp,
                                                 int32_t* s_dst) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int R = static_cast<int>(gridDim.x) * top_k;
  const int r0 = static_cast<int>(row) * top_k;
  // this kernel starts the call: CTA 0 clears the status words (the
  // bad-id count it adds to below, the GEMMs' error word)
  if (status && blockIdx.x == 0 && tid < 2) status[tid] = 0u;
  for (int e = tid; e <= E; e += blockDim.x) s_off[e] = 0;
  for (int i = tid; i < top_k; i += blockDim.x) {
    s_rank[i] = 0;
    s_exp[i] = id_of(r0 + i);
  }
  __syncthreads();
  int32_t mine[kInlinePer];
  uint32_t bad = 0;
#pragma unroll
  for (int j = 0; j < kInlinePer; ++j) {
    const int r = tid + j * static_cast<int>(blockDim.x);
    const int32_t e = r < R ? id_of(r) : -1;
    mine[j] = e;
    if (e >= 0 && e < E) atomicAdd(&s_off[e], 1);
    else if (e != -1) ++bad;
  }
  if (bad && blockIdx.x == 0 && status) atomicAdd(status, bad);
  // rank of each of the token's routes among the earlier routes of its expert
  for (int i = 0; i < top_k; ++i) {
    const int32_t e = s_exp[i];  // the same for every thread of the CTA
    if (e < 0 || e >= E) continue;
    int c = 0;
#pragma unroll
    for (int j = 0; j < kInlinePer; ++j)
      c += (mine[j] == e && tid + j * static_cast<int>(blockDim.x) < r0 + i) ? 1 : 0;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) c += __shfl_xor_sync(0xffffffffu, c, d);
    if (lane == 0 && c) atomicAdd(&s_rank[i], c);
  }
  __syncthreads();
  // exclusive scan of the counts in place: s_off[e] = first slot of expert e,
  // s_off[E] = valid routes
  if (tid < 32) {
    int32_t carry = 0;
    for (int e0 = 0; e0 <= E; e0 += 32) {
      const int e = e0 + lane;
      const int32_t v = e < E ? s_off[e] : 0;
      int32_t incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += n;
      }
      if (e <= E) s_off[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
  for (int i = tid; i < top_k; i += blockDim.x) {
    const int32_t e = s_exp[i];
    const int32_t slot = (e >= 0 && e < E) ? s_off[e] + s_rank[i] : -1;
    s_dst[i] = slot;
    slot_of[r0 + i] = slot;
    if (slot >= 0) sorted[slot] = r0 + i;
  }
  if (blockIdx.x == 0) {
    for (int e = tid; e < E; e += blockDim.x) {
      counts[e] = s_off[e + 1] - s_off[e];
      offsets[e] = s_off[e];
    }
    if (tid == 0) offsets[E] = s_off[E];
  }
  __syncthreads();
}

__device__ __forceinline__ void inline_route_slots(const InlinePlan& plan, int64_t row, int top_k,
                                                   int32_t* s_off, int32_t* s_rank, int32_t* s_exp,
                                                   int32_t* s_dst) {
  const int32_t* ids = plan.ids;
  plan_route_slots([ids](int r) { return ids[r]; }, plan.E, row, top_k, plan.counts,
                   plan.offsets, plan.sorted, plan.slot_of, plan.status, s_off, s_rank, s_exp,
                   s_dst);
}

// gstatic != nullptr (W4A4 with static activation globals, NT = 1): the
// block of each destination slot is quantised under gstatic[e] of that
// slot's expert e (token mode: eids[row * top_k + k]; row mode:
// eids[sorted[row]]) and its g is 1, because the GEMM epilogue then scales by
// the caller's per-expert alpha. Otherwise the row's global is dynamic,
// G0 = 448 * 6 / max|row|, with NT terms at G0 * 4^t.
__global__ void __launch_bounds__(1024) split_nvfp4_kernel(
    const void* __restrict__ src, int src_dt, SplitRows rows, const int32_t* __restrict__ slot_of,
    int top_k, const int32_t* __restrict__ n_rows_dev, int K, int NT, uint8_t* __restrict__ q,
    uint8_t* __restrict__ sf, float* __restrict__ gout, const float* __restrict__ gstatic,
    const int32_t* __restrict__ eids, const int32_t* __restrict__ sorted, const InlinePlan plan,
    int64_t plane) {
  __shared__ float s_max[32];
  __shared__ int32_t s_dst[kMaxTopK];
  __shared__ int32_t s_off[kMaxExperts + 1];
  __shared__ int32_t s_rank[kMaxTopK];
  __shared__ int32_t s_exp[kMaxTopK];
  __shared__ int s_any;
  const int64_t row = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  if (n_rows_dev && row >= static_cast<int64_t>(*n_rows_dev)) return;
  const int tid = threadIdx.x;
  int ndst = 1;
  const bool token = slot_of != nullptr || plan.ids != nullptr;  // token mode
  if (token) {
    if (tid == 0) s_any = 0;
    if (plan.ids) {
      inline_route_slots(plan, row, top_k, s_off, s_rank, s_exp, s_dst);
      for (int i = tid; i < top_k; i += blockDim.x)
        if (s_dst[i] >= 0) s_any = 1;
    } else {
      __syncthreads();
      for (int i = tid; i < top_k; i += blockDim.x) {
        s_dst[i] = slot_of[row * top_k + i];
        if (s_dst[i] >= 0) s_any = 1;
      }
    }
    __syncthreads();
    if (!s_any) return;  // the whole CTA leaves together
    ndst = top_k;
  }
  const void* rsrc = src;
  int64_t rbase = row * K;
  if (rows.base) {
    rsrc = rows.base[row / rows.rows_per_src];
    rbase = (row % rows.rows_per_src) * K;
  }
  const int blk = tid;  // this thread's 16-element block
  const bool active = blk * 16 < K;
  float v[16];
  if (active) {
    if (rows.base) {
      load8<true>(rsrc, src_dt, rbase + blk * 16, v);
      load8<true>(rsrc, src_dt, rbase + blk * 16 + 8, v + 8);
    } else {
      load8(rsrc, src_dt, rbase + blk * 16, v);
      load8(rsrc, src_dt, rbase + blk * 16 + 8, v + 8);
    }
  }
  if (gstatic) {
    for (int d = 0; d < ndst; ++d) {
      const int64_t dst = token ? static_cast<int64_t>(s_dst[d]) : row;
      if (dst < 0) continue;
      const int32_t e = token ? eids[row * top_k + d] : eids[sorted[row]];
      const float G = gstatic[e];
      if (tid == 0) gout[dst] = 1.0f;
      if (!active) continue;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = v[i];
      uint32_t w[2];
      uint8_t s8;
      quant_block<false>(x, G, __fdiv_rn(1.0f, G), w, &s8);
      *reinterpret_cast<uint2*>(q + dst * (K / 2) + blk * 8) = make_uint2(w[0], w[1]);
      sf[dst * (K / 16) + blk] = s8;
    }
    return;
  }
  split_row_terms(v, active, NT, K, token ? s_dst : nullptr, ndst, row, q, sf, gout, s_max,
                  plane);
}

// Expert-parallel exchange split (EpSplitArgs): one CTA per virtual token
// v = src * max_tokens + t of the whole world's step, blockDim as the split.
//  1. The CTAs of this rank's own tokens copy their row, ids and weights into
//     the exchange buffer; after a CTA barrier one thread per CTA fences at
//     system scope and counts the CTA done, and the last of them raises
//     ready = epoch << 32 | M on every other rank.
//  2. Every CTA waits (bounded) for the other ranks' ready flags, reads every
//     rank's ids (its own from the caller, the others' over NVLink), keeps
//     the routes to this rank's experts and plans their slots in the stable
//     (expert, virtual route) order, like the single-GPU in-split plan.
//  3. A CTA whose token has a local route reads the row (from the caller, or
//     from the source GPU through L2 only) and splits it into its slots.
// The publishing CTAs raise the flag before they wait, and the waiting CTAs
// need nothing from this rank's publishers, so the grid completes even when
// it is not all resident at once.
__global__ void __launch_bounds__(1024) ep_split_kernel(
    const EpSplitArgs a, int src_dt, int top_k, int K, int NT, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets, int32_t* __restrict__ sorted, int32_t* __restrict__ slot_of,
    uint32_t* __restrict__ status, uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
    float* __restrict__ gout) {
  __shared__ float s_max[32];
  __shared__ int32_t s_dst[kMaxTopK];
  __shared__ int32_t s_off[kMaxExperts + 1];
  __shared__ int32_t s_rank[kMaxTopK];
  __shared__ int32_t s_exp[kMaxTopK];
  __shared__ int64_t s_cnt[kMaxWorld];
  __shared__ int s_any;
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  const int64_t v = blockIdx.x;
  const int src = static_cast<int>(v / a.max_tokens);
  const int64_t t = v - static_cast<int64_t>(src) * a.max_tokens;
  const EpTables* tab = a.tab;
  const unsigned long long epoch = a.dev->epoch;
  if (v == 0 && tid < 2) status[tid] = 0u;  // bad-id count, error word of this call
  // 1. publish this rank's tokens
  const int64_t publishers = a.M > 0 ? a.M : 1;
  if (src == a.rank && t < publishers) {
    if (t < a.M) {
      const int64_t vec = static_cast<int64_t>(K) * a.act_bytes / 16;
      const uint4* from = static_cast<const uint4*>(a.hidden) + t * vec;
      uint4* to = static_cast<uint4*>(a.ex_hidden) + t * vec;
      for (int64_t i = tid; i < vec; i += blockDim.x) to[i] = from[i];
      for (int i = tid; i < top_k; i += blockDim.x) {
        a.ex_ids[t * top_k + i] = a.ids[t * top_k + i];
        a.ex_weights[t * top_k + i] = a.weights[t * top_k + i];
      }
    }
    // the barrier orders every thread's copies before thread 0's
    // system-scope fence (cumulative), which orders them before the count
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      const unsigned int done = atomicAdd(&a.dev->publish_count, 1u) + 1u;
      if (done == static_cast<unsigned int>(publishers)) {
        a.dev->publish_count = 0u;
        __threadfence_system();
        const unsigned long long val = (epoch << 32) | static_cast<unsigned long long>(a.M);
        for (int d = 0; d < a.world; ++d)
          if (d != a.rank) st_release_sys(tab->ready_at_peer[d], val);
      }
    }
  }
  // 2. every rank's token count, then the plan of the local routes
  const uint64_t deadline = globaltimer_ns() + kEpWaitNs;
  for (int s2 = tid; s2 < a.world; s2 += blockDim.x) {
    unsigned long long seen = 0;
    if (s2 == a.rank) {
      s_cnt[s2] = a.M;
    } else {
      s_cnt[s2] = ep_wait_epoch(&a.ready[s2], epoch, true, &seen, &a.dev->errors, deadline)
                      ? static_cast<int64_t>(seen & 0xffffffffull)
                      : 0;
    }
  }
  __syncthreads();
  const int e_lo = tab->shard_begin[a.rank];
  const int e_hi = tab->shard_begin[a.rank + 1];
  const int64_t mt = a.max_tokens;
  const int rank = a.rank;
  const int32_t* own_ids = a.ids;
  auto id_of = [&](int r) -> int32_t {
    const int64_t vv = r / top_k;
    const int ss = static_cast<int>(vv / mt);
    const int64_t tt = vv - static_cast<int64_t>(ss) * mt;
    if (tt >= s_cnt[ss]) return -1;
    const int64_t at = tt * top_k + (r - vv * top_k);
    const int32_t e = ss == rank ? own_ids[at] : __ldcg(tab->peer_ids[ss] + at);
    return (e >= e_lo && e < e_hi) ? e - e_lo : -1;
  };
  plan_route_slots(id_of, e_hi - e_lo, v, top_k, counts, offsets, sorted, slot_of, nullptr,
                   s_off, s_rank, s_exp, s_dst);
  // 3. the token's row into its slots
  if (t >= s_cnt[src]) return;  // the whole CTA leaves together
  if (tid == 0) s_any = 0;
  __syncthreads();
  for (int i = tid; i < top_k; i += blockDim.x)
    if (s_dst[i] >= 0) s_any = 1;
  __syncthreads();
  if (!s_any) return;
  const bool active = tid * 16 < K;
  float x[16];
  if (active) {
    const int64_t at = t * K + tid * 16;
    if (src == a.rank) {
      load8(a.hidden, src_dt, at, x);
      load8(a.hidden, src_dt, at + 8, x + 8);
    } else {
      load8<true>(tab->peer_hidden[src], src_dt, at, x);
      load8<true>(tab->peer_hidden[src], src_dt, at + 8, x + 8);
    }
  }
  split_row_terms(x, active, NT, K, s_dst, top_k, 0, q, sf, gout, s_max);
}

// ---- host ---------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool encode_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
               uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Three-dimensional u8 map of NT term planes [planes][rows][inner] (plane
// stride rows * inner bytes), box {box_inner, box_rows, planes}.
bool encode_u8_planes(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                      uint64_t planes, uint32_t box_inner, uint32_t box_rows,
                      CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (!fn) return false;
  const cuuint64_t dims[3] = {inner, rows, planes};
  const cuuint64_t strides[2] = {inner, inner * rows};
  const cuuint32_t box[3] = {box_inner, box_rows, static_cast<cuuint32_t>(planes)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, int BNR, int NT, bool KT>
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& sa, const CUtensorMap& b,
                        const CUtensorMap& sb, const BsParams& p, int grid, cudaStream_t stream) {
  using C = BsCfg<MODE, BNR, NT, KT>;
  auto kern = moe_gemm_bs_kernel<MODE, BNR, NT, KT>;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  // once per device and instantiation; a repeat from a racing thread is harmless
  static std::atomic<bool> attr[64] = {};
  if (dev < 0 || dev >= 64 || !attr[dev].load(std::memory_order_acquire)) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) attr[dev].store(true, std::memory_order_release);
  }
  return launch_kernel(true, kern, dim3(grid), dim3(kThreads), C::kSmem, stream, a, sa, b, sb, p);
}

template <int MODE, int NT>
cudaError_t launch_bnr_nt(int bnr, const CUtensorMap& a, const CUtensorMap& sa,
                          const CUtensorMap& b, const CUtensorMap& sb, const BsParams& p, int grid,
                          cudaStream_t stream) {
  switch (bnr) {
    case 16: return launch_gemm<MODE, 16, NT, false>(a, sa, b, sb, p, grid, stream);
    case 32: return launch_gemm<MODE, 32, NT, false>(a, sa, b, sb, p, grid, stream);
    case 64: return launch_gemm<MODE, 64, NT, false>(a, sa, b, sb, p, grid, stream);
    case 96: return launch_gemm<MODE, 96, NT, false>(a, sa, b, sb, p, grid, stream);
    case 128: return launch_gemm<MODE, 128, NT, false>(a, sa, b, sb, p, grid, stream);
    case 192: return launch_gemm<MODE, 192, NT, false>(a, sa, b, sb, p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

// nt = 4: bf16/f16/f32 activations as four NVFP4 terms (W4A16 results);
// nt = 1: activations quantised once (W4A4). kt: kKtTerms term planes run
// along K (N = bnr tokens), W4A16 at prefill sizes.
template <int MODE>
cudaError_t launch_bnr(const BsTile& tile, int nt, const CUtensorMap& a, const CUtensorMap& sa,
                       const CUtensorMap& b, const CUtensorMap& sb, const BsParams& p, int grid,
                       cudaStream_t stream) {
  if (tile.kt) {
    if (nt != kKtTerms) return cudaErrorInvalidValue;
    switch (tile.bnr) {
      case 64: return launch_gemm<MODE, 64, kKtTerms, true>(a, sa, b, sb, p, grid, stream);
      case 80: return launch_gemm<MODE, 80, kKtTerms, true>(a, sa, b, sb, p, grid, stream);
      case 128: return launch_gemm<MODE, 128, kKtTerms, true>(a, sa, b, sb, p, grid, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  if (nt == kSplitTerms)
    return launch_bnr_nt<MODE, kSplitTerms>(tile.bnr, a, sa, b, sb, p, grid, stream);
  if (nt == 1) return launch_bnr_nt<MODE, 1>(tile.bnr, a, sa, b, sb, p, grid, stream);
  return cudaErrorInvalidValue;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// slot_of != nullptr or plan->ids != nullptr: token mode (n_rows source
// tokens, terms scattered to their route slots); otherwise n_rows rows
// (device count n_rows_dev when given, n_rows an upper bound). The plan
// (token rows on this GPU, n_rows * top_k <= kInlinePlanRoutes) makes the
// split the first kernel of the call, so it is launched without PDL.
cudaError_t launch_split(const void* src, int src_dt, const SplitRows* rows,
                         const int32_t* slot_of, int top_k, const int32_t* n_rows_dev,
                         int64_t n_rows, int K, int nt, uint8_t* q, uint8_t* sf, float* g,
                         const float* gstatic, const int32_t* eids, const int32_t* sorted,
                         cudaStream_t stream, const InlinePlan* plan = nullptr,
                         int64_t plane = 0) {
  if (n_rows <= 0) return cudaSuccess;
  const SplitRows r = rows ? *rows : SplitRows{nullptr, 1};
  const InlinePlan ip = plan ? *plan : InlinePlan{};
  if (ip.ids && (r.base || n_rows * top_k > kInlinePlanRoutes || ip.E > kMaxExperts))
    return cudaErrorInvalidValue;
  if (K % 16 != 0 || K / 16 > 1024) return cudaErrorInvalidValue;
  // one CTA per row (rows on another GPU then cross NVLink once)
  const int threads = std::max(kSplitThreads, (K / 16 + 31) / 32 * 32);
  const dim3 grid(static_cast<unsigned>(n_rows));
  return launch_kernel(ip.ids == nullptr, split_nvfp4_kernel, grid, dim3(threads), 0, stream, src,
                       src_dt, r, ip.ids ? nullptr : slot_of, top_k, n_rows_dev, K, nt, q, sf, g,
                       gstatic, eids, sorted, ip, plane);
}

}  // namespace

cudaError_t read_sticky_errors(cudaStream_t stream, uint32_t* errors) {
  cudaError_t err = cudaMemcpyFromSymbolAsync(errors, g_sticky_errors, sizeof(uint32_t), 0,
                                              cudaMemcpyDeviceToHost, stream);
  if (err != cudaSuccess) return err;
  err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return err;
  const uint32_t zero = 0;
  err = cudaMemcpyToSymbolAsync(g_sticky_errors, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                                stream);
  if (err != cudaSuccess) return err;
  return cudaStreamSynchronize(stream);
}

uint64_t set_kernel_wait_ns(uint64_t ns) {
  return g_wait_ns.exchange(ns ? ns : kTimeoutNs, std::memory_order_relaxed);
}

bool bs_supported(int K, int I) {
  return K % kBK == 0 && I % kBK == 0 && K <= 16384 && I <= 16384 && get_encode() != nullptr;
}

// Term rows per MMA tile: enough for ~1.5x the mean routes per expert, up to
// 32 tokens (from N = 128 the block-scaled MMA runs at full rate; below N =
// 64 it costs a fixed ~46 cycles per instruction). When experts see more
// tokens than that (prefill), the terms go along K instead (kt): N = 128
// tokens per gate/up tile (one accumulator buffer) and 64 per down tile (two
// buffers, so a unit's epilogue overlaps the next unit's MMAs, which matters
// with only I / 256 K stages per unit). Per byte of weights staged a tile
// then serves 128 (64) tokens instead of 48 (24); each token brings its four
// term planes, so the bytes staged per MMA cycle drop by about a third.
BsTile bs_tile(int64_t routes, int E, int mode, int nt) {
  const double per_expert = static_cast<double>(routes) / E;
  if (nt == kSplitTerms && routes > kInlinePlanRoutes && per_expert >= kKtMinTokens)
    return {mode == kGateUp ? 128 : 80, true};
  const double want = per_expert * 1.5 * nt;  // term rows
  int rows = 16;
  while (rows < want && rows < 128) rows *= 2;
  if (rows == 128 && want > 192.0) return {mode == kGateUp ? 192 : 96, false};
  return {rows, false};
}

cudaError_t launch_moe_bs(const BsLaunch& a, cudaStream_t stream, const char** step) {
  const int64_t R = a.R;
  const int NT = a.nt;
  const bool w4a4_static = a.a13_gscale != nullptr;
  const int grid = sm_count();
  const uint64_t brows = static_cast<uint64_t>(R > 0 ? R : 1) * NT;
  // All tensor maps are encoded before the first launch, so the host never
  // holds the stream up between kernels.
  *step = "tensor maps";
  const BsTile tile1 = bs_tile(R, a.E, kGateUp, NT);
  const BsTile tile2 = bs_tile(R, a.E, kDown, NT);
  // the exchange split (at most kInlinePlanRoutes routes) writes the rows layout
  if (a.ep && tile1.kt) return cudaErrorInvalidValue;
  // K layout: kKtTerms planes of R rows each (inside the workspace's R * NT rows)
  const uint64_t plane_rows = static_cast<uint64_t>(R > 0 ? R : 1);
  const int64_t plane1 = tile1.kt ? static_cast<int64_t>(plane_rows) : 0;
  const int64_t plane2 = tile2.kt ? static_cast<int64_t>(plane_rows) : 0;
  const int nt1 = tile1.kt ? kKtTerms : NT;
  const int nt2 = tile2.kt ? kKtTerms : NT;
  auto encode_b = [&](CUtensorMap* m, CUtensorMap* ms, const void* q, const void* sf, int k,
                      const BsTile& t) {
    if (t.kt)
      return encode_u8_planes(m, q, k / 2, plane_rows, kKtTerms, kRowBytes, t.bnr,
                              CU_TENSOR_MAP_SWIZZLE_128B) &&
             encode_u8_planes(ms, sf, k / 16, plane_rows, kKtTerms, kRowScales, t.bnr,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
    return encode_u8(m, q, k / 2, brows, kRowBytes, t.bnr, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_u8(ms, sf, k / 16, brows, kRowScales, t.bnr, CU_TENSOR_MAP_SWIZZLE_NONE);
  };
  CUtensorMap m1a, m1sa, m1b, m1sb, m2a, m2sa, m2b, m2sb;
  if (!encode_u8(&m1a, a.w13, a.K / 2, (uint64_t)a.E * 2 * a.I, kRowBytes, kM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_u8(&m1sa, a.s13, a.K / 16, (uint64_t)a.E * 2 * a.I, kRowScales, kM,
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_b(&m1b, &m1sb, a.xq, a.xsf, a.K, tile1) ||
      !encode_u8(&m2a, a.w2, a.I / 2, (uint64_t)a.E * a.K, kRowBytes, kM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_u8(&m2sa, a.s2, a.I / 16, (uint64_t)a.E * a.K, kRowScales, kM,
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_b(&m2b, &m2sb, a.hq, a.hsf, a.I, tile2))
    return cudaErrorInvalidValue;
  BsParams p1{};
  p1.counts = a.counts;
  p1.offsets = a.offsets;
  // static W4A4: the caller's per-expert alpha scales the MMA result alone
  p1.gscale = w4a4_static ? a.alpha13 : a.g13;
  p1.bg = a.xg;
  p1.out = a.h;
  p1.status = a.status;
  p1.E = a.E;
  p1.I = a.I;
  p1.m_tiles = a.I / kM;
  p1.a_stride = a.I;
  p1.k_stages = a.K / kBK;
  p1.rows_per_expert = 2 * a.I;
  p1.out_ld = a.I;
  // about one token tile per expert: every weight tile is read once
  p1.stream_weights = R <= static_cast<int64_t>(a.E) * (tile1.kt ? tile1.bnr : tile1.bnr / NT);
  p1.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  p1.bsf = a.xsf;
  p1.plane = plane1;
  // a call whose plan the activation split computes: both GEMMs derive it
  // from the ids themselves and start streaming weights before the split ends
  p1.early_ids = (a.inline_plan && !a.ep && !a.hidden_rows.base) ? a.ids : nullptr;
  p1.wa = a.w13;
  p1.wa_ld = a.K / 2;
  // gate/up tiles keep the TMA alone: with the split, their prefill launches
  // measured 2.5 % slower (1.418 against 1.383 ms, T = 8192, same clocks)
  p1.lsu_half = false;
  p1.early_routes = static_cast<int>(R);
  BsParams p2 = p1;
  p2.gscale = w4a4_static ? a.alpha2 : a.g2;
  p2.bg = a.hg;
  p2.out = a.y;
  p2.m_tiles = a.K / (2 * kM);
  p2.a_stride = kM;
  p2.k_stages = a.I / kBK;
  p2.rows_per_expert = a.K;
  p2.out_ld = a.K;
  p2.stream_weights = R <= static_cast<int64_t>(a.E) * (tile2.kt ? tile2.bnr : tile2.bnr / NT);
  p2.bsf = a.hsf;
  p2.plane = plane2;
  p2.wa = a.w2;
  p2.wa_ld = a.I / 2;
  p2.lsu_half = !p2.stream_weights;

  if (a.push.base) {
    // expert parallel: rows go back to their source ranks, unweighted
    p2.push_base = a.push.base;
    p2.push_rows = a.push.rows_per_src;
    p2.sorted = a.sorted;
    p2.top_k = a.top_k;
  }

  // 1. split each token once; its terms go to all of its route slots (for a
  //    small call the split also computes the route plan, and in an
  //    expert-parallel step it also exchanges the step with the other ranks)
  *step = "activation split";
  cudaError_t err = cudaSuccess;
  if (a.ep) {
    if (a.K % 16 != 0 || a.K / 16 > 1024 || a.M * a.top_k > kInlinePlanRoutes ||
        a.a13_gscale || a.E > kMaxExperts)
      return cudaErrorInvalidValue;
    const int threads = std::max(kSplitThreads, (a.K / 16 + 31) / 32 * 32);
    err = launch_kernel(true, ep_split_kernel, dim3(static_cast<unsigned>(a.M)), dim3(threads), 0,
                        stream, *a.ep, a.act_dt, a.top_k, a.K, NT, a.counts, a.offsets, a.sorted,
                        a.slot_of, a.status, a.xq, a.xsf, a.xg);
  } else {
    const InlinePlan plan{a.inline_plan ? a.ids : nullptr, a.E, a.counts, a.offsets, a.sorted,
                          a.slot_of, a.status};
    err = launch_split(a.hidden, a.act_dt, &a.hidden_rows, a.slot_of, a.top_k, nullptr, a.M, a.K,
                       nt1, a.xq, a.xsf, a.xg, a.a13_gscale, a.ids, a.sorted, stream, &plan,
                       plane1);
  }
  if (err != cudaSuccess) return err;
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 1);
  // 2. gate/up + SwiGLU
  *step = "gate/up";
  err = launch_bnr<kGateUp>(tile1, nt1, m1a, m1sa, m1b, m1sb, p1, grid, stream);
  if (err != cudaSuccess) return err;
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 2);
  // 3. split the SwiGLU rows, down projection
  *step = "h split";
  err = launch_split(a.h, kF32, nullptr, nullptr, 1, a.offsets + a.E, R, a.I, nt2, a.hq, a.hsf,
                     a.hg, a.a2_gscale, a.ids, a.sorted, stream, nullptr, plane2);
  if (err != cudaSuccess) return err;
  *step = "down";
  err = launch_bnr<kDown>(tile2, nt2, m2a, m2sa, m2b, m2sb, p2, grid, stream);
  if (err != cudaSuccess) return err;
  if (a.stage_mark) a.stage_mark(a.stage_ctx, 3);
  return cudaSuccess;
}

}  // namespace sbb
