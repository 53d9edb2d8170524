// Workspace plan and kernel-choice driver for one routed-expert MoE call.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "kernels.h"

namespace sbb {

constexpr size_t kStatusOffset = 0;  // uint32 status words at the workspace start

// Byte offsets of each region inside the caller's workspace. The size query
// and the launcher both derive them from plan_workspace, so they cannot drift
// (the reference's plan_workspace rule, nvfp4_moe_grouped.sycl.cpp:92-130).
struct WorkspacePlan {
  size_t status;        // uint32[64]: [0] ids outside [-1, E)
  size_t chunk_counts;  // int32[nchunks * E]
  size_t counts;        // int32[E]
  size_t offsets;       // int32[E + 1]
  size_t sorted;        // int32[R]   route id per sorted slot
  size_t slot_of;       // int32[R]   sorted slot per route, -1 if dropped
  size_t h;             // fp32[R, I] SwiGLU activations per slot
  size_t xq, xsf, xg;   // activation split terms: [R*NT, K/2], [R*NT, K/16], fp32 [R*NT]
  size_t hq, hsf, hg;   // SwiGLU split terms:     [R*NT, I/2], [R*NT, I/16], fp32 [R*NT]
  size_t y;             // fp32[R, K] down-projection output per slot
  size_t total;
};

WorkspacePlan plan_workspace(size_t M, size_t E, size_t top_k, size_t K, size_t I);
size_t route_plan_scratch_bytes(size_t routes, size_t E);

struct MoeArgs {
  const void* hidden;
  int act_dt;
  const int32_t* ids;
  const float* weights;
  int multiply_router_weight;
  const uint8_t *w13, *s13, *w2, *s2;
  const float *g13, *g2;
  void* out;
  int out_dt;
  int64_t M;
  int E, top_k, K, I;
  void* const* stage_events;  // optional cudaEvent_t[SBB200_STAGE_EVENTS]
  // expert parallel (block-scaled path only): token rows read from the
  // source GPUs (hidden_rows) or the whole exchange done by the activation
  // split (ep_split; M is then the number of virtual tokens), and the down
  // projection's fp32 rows pushed back to their sources (push; no combine)
  SplitRows hidden_rows{nullptr, 1};
  const EpSplitArgs* ep_split = nullptr;
  PushRows push{nullptr, 1};
  // routing from router logits [M, E] (logits_dt): the plan writes top-k ids
  // into `routed_ids` and softmax weights into `routed_weights`, which the
  // rest of the forward then uses in place of ids / weights
  // activation terms: kSplitTerms (W4A16 results) or 1 (W4A4: one NVFP4
  // quantisation of the activations, dynamic per row unless a13_gscale is
  // set, in which case a13/a2_gscale quantise and alpha13/alpha2 scale)
  int act_terms = kSplitTerms;
  const float *a13_gscale = nullptr, *a2_gscale = nullptr;
  const float *alpha13 = nullptr, *alpha2 = nullptr;
  const void* router_logits = nullptr;
  int logits_dt = 0;
  int32_t* routed_ids = nullptr;
  float* routed_weights = nullptr;
};

int validate_shape(size_t M, size_t E, size_t top_k, size_t K, size_t I, int act_dt, int out_dt,
                   std::string* why);

// True when the activation split computes the route plan itself (no plan
// kernel): a small call (R = M * top_k routes, at most kInlinePlanRoutes) on
// the block-scaled path, token rows on this GPU, ids given rather than routed
// from logits.
bool plan_in_split(int64_t R, int K, int I, bool rows_local, bool from_logits);

// Kernels (excluding the status memset) one run_moe call enqueues when ids
// are given; rows_local is false for expert-parallel rows read from peers.
int count_launches(int64_t M, int top_k, int K, int I, bool rows_local = true);

// True when an expert-parallel step of world * max_tokens virtual tokens is
// exchanged by the activation split itself (ep_split_kernel).
bool ep_split_fits(int64_t virtual_tokens, int top_k, int K, int I, int E_local);

// Enqueue the whole forward on `stream`. On failure returns the CUDA error and
// names the failing step in *why.
cudaError_t run_moe(const MoeArgs& a, const WorkspacePlan& plan, void* workspace,
                    cudaStream_t stream, std::string* why);

}  // namespace sbb
