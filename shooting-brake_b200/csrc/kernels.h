// Host-side launch entry points of the device kernels (internal to the
// library; the public surface is include/sbb200.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace sbb {

constexpr int kRouteChunk = 4096;  // routes per CTA in the route plan
// Up to this many routes (M * top_k) on the block-scaled path with token rows
// on this GPU, the activation split computes the route plan itself.
constexpr int kInlinePlanRoutes = 1024;

// Sets the calling thread's message returned by sbb200_last_error.
void set_last_error(const std::string& msg);
constexpr int kMaxExperts = 512;   // route-plan shared-memory bound
constexpr int kMaxTopK = 64;

size_t route_plan_chunks(int64_t R);
size_t route_scatter_smem(int E);

// With `logits` ([R / top_k, E] in logits_dt) the plan first routes every
// token (top-k + softmax) into `ids` (then written, not read) and `weights`;
// a single-chunk plan does it inside its one CTA.
cudaError_t launch_route_plan(const int32_t* ids, int64_t R, int E, int32_t* chunk_counts,
                              int32_t* counts, int32_t* offsets, int32_t* sorted,
                              int32_t* slot_of, uint32_t* status, cudaStream_t stream,
                              const void* logits = nullptr, int logits_dt = 0, int top_k = 1,
                              float* weights = nullptr);

// Top-k routing: ids int32 [M, k], weights fp32 [M, k] from logits [M, E].
cudaError_t launch_router_topk(const void* logits, int dt, int64_t M, int E, int k, int32_t* ids,
                               float* weights, cudaStream_t stream);

// CUDA-core grouped expert kernels: any K, I that are multiples of 32.
// h: fp32 [R, I] in sorted-slot order; y: fp32 [R, K] (global scale applied,
// router weight not applied).
cudaError_t launch_gateup_simt(const void* hidden, int act_dt, int top_k, const uint8_t* w13,
                               const uint8_t* s13, const float* g13, const int32_t* counts,
                               const int32_t* offsets, const int32_t* sorted, float* h, int E,
                               int K, int I, cudaStream_t stream);
cudaError_t launch_down_simt(const float* h, const uint8_t* w2, const uint8_t* s2,
                             const float* g2, const int32_t* counts, const int32_t* offsets,
                             float* y, int E, int K, int I, cudaStream_t stream);

// Rows of a [world * rows_per_src, K] operand that live on different GPUs:
// row v is at base[v / rows_per_src] + (v % rows_per_src) * K elements.
struct SplitRows {
  const void* const* base;  // device array of per-source row bases (peer pointers)
  int64_t rows_per_src;
};

// ---- expert parallelism (ep.cu) ------------------------------------------
constexpr int kMaxWorld = 64;

// Peer addresses of one rank's exchange (device memory, filled at connect).
struct EpTables {
  unsigned long long* ready_at_peer[kMaxWorld];  // &peer.ready[rank]
  unsigned long long* done_at_peer[kMaxWorld];   // &peer.done[rank]
  const void* peer_hidden[kMaxWorld];
  const int32_t* peer_ids[kMaxWorld];
  const float* peer_weights[kMaxWorld];
  float* partial_at_peer[kMaxWorld];  // peer's partial [max_tokens, top_k, K] fp32
  int shard_begin[kMaxWorld + 1];
};

// Device-side state of one rank (local memory).
struct EpDev {
  unsigned long long epoch;   // epoch of the current step (bumped by the last
                              // CTA of the step's final kernel)
  unsigned int errors;        // bit 0: a wait for another rank timed out
  unsigned int final_count;   // CTAs of the final kernel done reading epoch
  unsigned int publish_count; // CTAs of the exchange split done publishing
  unsigned int pad[3];
};

constexpr uint64_t kEpWaitNs = 2000000000ull;  // 2 s per cross-GPU wait

// One expert-parallel step whose virtual routes (world * max_tokens *
// top_k) fit the in-kernel route plan: the activation split publishes this
// rank's tokens, raises its ready flag, waits for every rank's, plans the
// local routes and pulls the routed rows itself (no publish, gather or plan
// kernel).
struct EpSplitArgs {
  const EpTables* tab;               // device
  EpDev* dev;                        // device
  const unsigned long long* ready;   // this rank's ready flags [world]
  const void* hidden;                // this rank's tokens [M, K] (caller memory)
  const int32_t* ids;                // [M, top_k] global expert ids
  const float* weights;              // [M, top_k]
  void* ex_hidden;                   // this rank's exchange buffer regions
  int32_t* ex_ids;
  float* ex_weights;
  int world, rank, act_bytes;
  int64_t M, max_tokens;
};

// Down projection results pushed to their source ranks: route r = v * top_k
// + k of virtual token v = s * rows_per_src + t goes to row (t * top_k + k)
// of base[s] (fp32 [rows_per_src, top_k, K]).
struct PushRows {
  float* const* base;  // device array [world]
  int64_t rows_per_src;
};

// out[t, :] = sum over valid k of w[t, k] * y[slot_of[t*top_k + k], :], k ascending.
cudaError_t launch_combine(const float* y, const int32_t* slot_of, const float* weights,
                           int multiply_router_weight, void* out, int out_dt, int64_t M,
                           int top_k, int K, cudaStream_t stream);

// Bit-exact NVFP4 dequant: out[r, c] = e2m1 * fp32(e4m3 * g[r / rows_per_scale]).
cudaError_t launch_dequant(const uint8_t* q, const uint8_t* sf, const float* g,
                           int64_t rows_per_scale, float* out, int64_t rows, int64_t cols,
                           cudaStream_t stream);

// NVFP4 quantiser (vLLM ref_nvfp4_quant semantics) of a [rows, cols] matrix in
// dtype in_dt with per-group quantisation global gq[r / rows_per_scale].
cudaError_t launch_quantize(const void* x, int in_dt, const float* gq, int64_t rows_per_scale,
                            uint8_t* q, uint8_t* sf, int64_t rows, int64_t cols,
                            cudaStream_t stream);

// Block-scaled path (moe_bs.cu): activations split into kSplitTerms NVFP4
// terms, tcgen05.mma kind::mxf4nvf4 on the packed weights.
constexpr int kSplitTerms = 4;
// Bytes after a K-layout scale region: the contiguous scale run of a tile
// that ends past the last slot (at most 256 slots x 16 bytes) stays inside it.
constexpr size_t kScaleRunPad = 4096;

struct BsLaunch {
  const void* hidden;
  int act_dt;
  SplitRows hidden_rows;   // base != nullptr: token rows read from other GPUs
  int nt;                  // activation terms: kSplitTerms (W4A16) or 1 (W4A4)
  const int32_t* ids;      // route expert ids (static W4A4 global lookup)
  // static W4A4 (a13_gscale != nullptr): activation quantisation globals and
  // output scales per expert, vLLM's a1/a2_gscale and g1/g2_alphas
  const float *a13_gscale, *a2_gscale, *alpha13, *alpha2;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* slot_of;  // [M*top_k] sorted slot of each route, -1 if dropped
  // true: no route plan ran; the activation split writes counts, offsets,
  // sorted, slot_of and the bad-id count (status[0]) itself
  bool inline_plan;
  const uint8_t *w13, *s13, *w2, *s2;
  const float *g13, *g2;
  uint8_t* xq;   // [R*NT, K/2]
  uint8_t* xsf;  // [R*NT, K/16]
  float* xg;     // [R*NT]
  float* h;      // fp32 [R, I]
  uint8_t* hq;   // [R*NT, I/2]
  uint8_t* hsf;  // [R*NT, I/16]
  float* hg;     // [R*NT]
  float* y;      // fp32 [R, K]
  uint32_t* status;
  int64_t M, R;
  int E, top_k, K, I;
  void (*stage_mark)(void* ctx, int stage);
  void* stage_ctx;
  // expert parallel: the split exchanges the step itself (ep != nullptr;
  // M is then world * max_tokens virtual tokens) and/or the down projection
  // pushes its rows to the sources (push.base != nullptr, no y)
  const EpSplitArgs* ep = nullptr;
  PushRows push{nullptr, 1};
};

bool bs_supported(int K, int I);
// Sets the limit of the grouped GEMMs' pipeline waits for later launches (0:
// the 2 s default); returns the previous limit.
uint64_t set_kernel_wait_ns(uint64_t ns);
// Reads and clears the current device's sticky GEMM error bits (synchronises).
cudaError_t read_sticky_errors(cudaStream_t stream, uint32_t* errors);
// Token tile of one grouped GEMM: N = bnr (term rows, or tokens when kt),
// kt: the activation terms are planes along K (prefill-sized calls).
struct BsTile {
  int bnr;
  bool kt;
};
// mode: 0 gate/up, 1 down.
BsTile bs_tile(int64_t routes, int E, int mode, int nt);
cudaError_t launch_moe_bs(const BsLaunch& a, cudaStream_t stream, const char** step);

}  // namespace sbb
