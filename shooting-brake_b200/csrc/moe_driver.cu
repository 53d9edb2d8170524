// Kernel-choice driver: route plan -> gate/up + SwiGLU -> down -> combine.
#include "moe_driver.h"

#include "kernels.h"
#include "launch.cuh"

namespace sbb {

namespace {
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

size_t route_plan_scratch_bytes(size_t routes, size_t E) {
  return 256 + align_up(route_plan_chunks((int64_t)routes) * E * sizeof(int32_t), 256);
}

WorkspacePlan plan_workspace(size_t M, size_t E, size_t top_k, size_t K, size_t I) {
  const size_t R = M * top_k;
  WorkspacePlan p{};
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t here = at;
    at = align_up(at + bytes, 256);
    return here;
  };
  p.status = take(256);
  p.chunk_counts = take(route_plan_chunks((int64_t)R) * E * sizeof(int32_t));
  p.counts = take(E * sizeof(int32_t));
  p.offsets = take((E + 1) * sizeof(int32_t));
  p.sorted = take(R * sizeof(int32_t));
  p.slot_of = take(R * sizeof(int32_t));
  p.h = take(R * I * sizeof(float));
  const size_t RT = R * kSplitTerms;
  p.xq = take(RT * K / 2);
  // + one tile of K-layout scale runs read past the last slot
  p.xsf = take(RT * K / 16 + kScaleRunPad);
  p.xg = take(RT * sizeof(float));
  p.hq = take(RT * I / 2);
  p.hsf = take(RT * I / 16 + kScaleRunPad);
  p.hg = take(RT * sizeof(float));
  p.y = take(R * K * sizeof(float));
  p.total = at;
  return p;
}

bool ep_split_fits(int64_t virtual_tokens, int top_k, int K, int I, int E_local) {
  return virtual_tokens > 0 && virtual_tokens * top_k <= kInlinePlanRoutes &&
         E_local <= kMaxExperts && bs_supported(K, I);
}

bool plan_in_split(int64_t R, int K, int I, bool rows_local, bool from_logits) {
  return rows_local && !from_logits && R > 0 && R <= kInlinePlanRoutes && bs_supported(K, I);
}

int count_launches(int64_t M, int top_k, int K, int I, bool rows_local) {
  const int64_t R = M * top_k;
  const int plan = plan_in_split(R, K, I, rows_local, false) ? 0
                   : route_plan_chunks(R) > 1                 ? 2
                                                              : 1;
  // block-scaled path: activation split, gate/up, SwiGLU split, down;
  // CUDA-core path: gate/up, down. Both end with the combine.
  const int body = bs_supported(K, I) ? 4 : 2;
  return plan + body + 1;
}

cudaError_t run_moe(const MoeArgs& a, const WorkspacePlan& plan, void* workspace,
                    cudaStream_t stream, std::string* why) {
  char* ws = static_cast<char*>(workspace);
  auto* status = reinterpret_cast<uint32_t*>(ws + plan.status);
  auto* chunk_counts = reinterpret_cast<int32_t*>(ws + plan.chunk_counts);
  auto* counts = reinterpret_cast<int32_t*>(ws + plan.counts);
  auto* offsets = reinterpret_cast<int32_t*>(ws + plan.offsets);
  auto* sorted = reinterpret_cast<int32_t*>(ws + plan.sorted);
  auto* slot_of = reinterpret_cast<int32_t*>(ws + plan.slot_of);
  auto* h = reinterpret_cast<float*>(ws + plan.h);
  auto* y = reinterpret_cast<float*>(ws + plan.y);
  const int64_t R = a.M * a.top_k;
  auto mark = [&](int i) -> cudaError_t {
    if (!a.stage_events || !a.stage_events[i]) return cudaSuccess;
    return record_stage_event(static_cast<cudaEvent_t>(a.stage_events[i]), stream);
  };

  cudaError_t err = mark(0);
  if (err != cudaSuccess) { *why = "stage event"; return err; }
  if (a.ep_split && !bs_supported(a.K, a.I)) {
    *why = "expert-parallel exchange needs K and I multiples of 256";
    return cudaErrorInvalidValue;
  }
  const int32_t* ids = a.router_logits ? a.routed_ids : a.ids;
  const float* weights = a.router_logits ? a.routed_weights : a.weights;
  const bool inline_plan = plan_in_split(R, a.K, a.I, a.hidden_rows.base == nullptr,
                                         a.router_logits != nullptr);
  // a split that plans the routes itself, or exchanges the step, is the
  // call's first kernel and clears the status words; otherwise a memset does
  if (!a.ep_split && !inline_plan) {
    err = cudaMemsetAsync(status, 0, 256, stream);
    if (err != cudaSuccess) { *why = "status clear"; return err; }
  }
  if (!inline_plan && !a.ep_split) {
    err = launch_route_plan(ids, R, a.E, chunk_counts, counts, offsets, sorted, slot_of, status,
                            stream, a.router_logits, a.logits_dt, a.top_k, a.routed_weights);
    if (err != cudaSuccess) { *why = "route plan"; return err; }
  }
  if (bs_supported(a.K, a.I)) {
    BsLaunch t{};
    t.hidden = a.hidden;
    t.act_dt = a.act_dt;
    t.hidden_rows = a.hidden_rows;
    t.nt = a.act_terms;
    t.ids = ids;
    t.a13_gscale = a.a13_gscale;
    t.a2_gscale = a.a2_gscale;
    t.alpha13 = a.alpha13;
    t.alpha2 = a.alpha2;
    t.counts = counts;
    t.offsets = offsets;
    t.sorted = sorted;
    t.slot_of = slot_of;
    t.inline_plan = inline_plan;
    t.w13 = a.w13;
    t.s13 = a.s13;
    t.w2 = a.w2;
    t.s2 = a.s2;
    t.g13 = a.g13;
    t.g2 = a.g2;
    t.xq = reinterpret_cast<uint8_t*>(ws + plan.xq);
    t.xsf = reinterpret_cast<uint8_t*>(ws + plan.xsf);
    t.xg = reinterpret_cast<float*>(ws + plan.xg);
    t.h = h;
    t.hq = reinterpret_cast<uint8_t*>(ws + plan.hq);
    t.hsf = reinterpret_cast<uint8_t*>(ws + plan.hsf);
    t.hg = reinterpret_cast<float*>(ws + plan.hg);
    t.y = y;
    t.status = status;
    t.ep = a.ep_split;
    t.push = a.push;
    t.M = a.M;
    t.R = R;
    t.E = a.E;
    t.top_k = a.top_k;
    t.K = a.K;
    t.I = a.I;
    struct Ctx {
      void* const* ev;
      cudaStream_t s;
    } ctx{a.stage_events, stream};
    if (a.stage_events) {
      t.stage_mark = [](void* c, int i) {
        auto* x = static_cast<Ctx*>(c);
        if (x->ev[i]) record_stage_event(static_cast<cudaEvent_t>(x->ev[i]), x->s);
      };
      t.stage_ctx = &ctx;
    }
    const char* step = "block-scaled path";
    err = launch_moe_bs(t, stream, &step);
    if (err != cudaSuccess) { *why = step; return err; }
  } else {
    if (a.hidden_rows.base || a.push.base || a.act_terms != kSplitTerms) {
      *why = a.act_terms != kSplitTerms ? "W4A4 needs K and I multiples of 256"
                                        : "expert-parallel rows need K and I multiples of 256";
      return cudaErrorInvalidValue;
    }
    if ((err = mark(1)) != cudaSuccess) { *why = "stage event"; return err; }
    err = launch_gateup_simt(a.hidden, a.act_dt, a.top_k, a.w13, a.s13, a.g13, counts, offsets,
                             sorted, h, a.E, a.K, a.I, stream);
    if (err != cudaSuccess) { *why = "gate/up"; return err; }
    if ((err = mark(2)) != cudaSuccess) { *why = "stage event"; return err; }
    err = launch_down_simt(h, a.w2, a.s2, a.g2, counts, offsets, y, a.E, a.K, a.I, stream);
    if (err != cudaSuccess) { *why = "down"; return err; }
    if ((err = mark(3)) != cudaSuccess) { *why = "stage event"; return err; }
  }
  if (!a.push.base) {  // expert parallel: the sources sum the pushed rows
    err = launch_combine(y, slot_of, weights, a.multiply_router_weight, a.out, a.out_dt, a.M,
                         a.top_k, a.K, stream);
    if (err != cudaSuccess) { *why = "combine"; return err; }
  }
  if ((err = mark(4)) != cudaSuccess) { *why = "stage event"; return err; }
  return cudaSuccess;
}

}  // namespace sbb
