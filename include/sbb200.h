/*
 * sbb200 -- B200-native routed-expert NVFP4 MoE: the C-ABI boundary.
 *
 * Plain C: opaque handles, plain pointers and sizes, no torch types. Device
 * pointers are CUDA device addresses of the current device; `stream` is a
 * cudaStream_t passed as void*. Every compute entry point is stream-ordered
 * and never synchronises the host.
 *
 * Return convention (src/phase7/b70_capi.h:10 of the reference):
 *   0 = ok, >0 = busy, <0 = error. The error text of the calling thread's
 *   last failing call is available through sbb200_last_error().
 *
 * Weight layout is the reference op's (src/QuixiCore-XPU/include/quixicore/
 * xpu/ops.hpp:269-279): w13 [E, 2I, K/2] packed e2m1 (gate rows [0, I), up
 * rows [I, 2I), low nibble = even k), w13_scales [E, 2I, K/16] e4m3,
 * w13_global_scales fp32 [E] (the dequant multiplier), w2 [E, K, I/2],
 * w2_scales [E, K, I/16], w2_global_scales fp32 [E]. K is the hidden size.
 */
#ifndef SBB200_H
#define SBB200_H

#ifdef __cplusplus
#include <cstddef>
#include <cstdint>
extern "C" {
#else
#include <stddef.h>
#include <stdint.h>
#endif

#define SBB200_ABI_VERSION 1

/* Activation / output dtypes; the values of the reference's DType
 * {f32, f16, bf16} (src/QuixiCore-XPU/include/quixicore/xpu/runtime.hpp:21-27). */
enum sbb200_dtype { SBB200_F32 = 0, SBB200_F16 = 1, SBB200_BF16 = 2 };

enum sbb200_status {
  SBB200_OK = 0,
  SBB200_BUSY = 1,
  SBB200_EINVAL = -1,       /* bad pointer, shape, dtype or id range */
  SBB200_EWORKSPACE = -2,   /* workspace smaller than the size query */
  SBB200_ECUDA = -3,        /* a CUDA runtime call failed */
  SBB200_EUNSUPPORTED = -4, /* shape outside what the kernels implement */
  SBB200_ENOTLOADED = -5    /* provider layer not registered */
};

/* Monotonic ABI version (src/phase7/b70_capi.h:47-52). */
size_t sbb200_abi_version(void);

/* Copy the calling thread's last error message. Returns the length needed
 * including the NUL; writes a NUL-terminated prefix when buf is too small
 * (src/phase7/b70_capi.h:159-172 shape). */
size_t sbb200_last_error(char* buf, size_t size);

/* ---------------------------------------------------------------------------
 * Stateless operator: the drop-in for ops::nvfp4_moe_grouped and the PyTorch
 * extension op nvfp4_moe (src/QuixiCore-XPU/include/quixicore/xpu/ops.hpp:
 * 333-372, src/QuixiCore-XPU/src/dispatch/moe.cpp:80-134,
 * src/QuixiCore-XPU/bindings/pytorch/tk_xpu_ext.sycl:296-410).
 * ------------------------------------------------------------------------- */

/* Device workspace bytes sbb200_nvfp4_moe needs for this shape
 * (ops::nvfp4_moe_grouped_workspace_bytes, ops.hpp:363-366). */
size_t sbb200_nvfp4_moe_workspace_bytes(size_t M, size_t E, size_t top_k, size_t K, size_t I,
                                        int act_dt);

/* Number of kernels one sbb200_nvfp4_moe call of this shape launches on
 * its stream (the status clear, a memset, is not counted). No counterpart in
 * the reference; it lets a benchmark or a graph builder account for launches. */
int sbb200_nvfp4_moe_launches(size_t M, size_t E, size_t top_k, size_t K, size_t I,
                              int act_dt);

/* out[M, K] = sum_k w[m, k] * FFN_{ids[m, k]}(hidden[m]) with
 * FFN(x) = W2 (silu(W_gate x) * (W_up x)). hidden [M, K] in act_dt (f32, f16
 * or bf16); topk_ids int32 [M, top_k], ids outside [0, E) are skipped (their
 * count is kept, see sbb200_nvfp4_moe_bad_ids); topk_weights fp32 [M, top_k]
 * (ignored when multiply_router_weight is 0). out [M, K] in out_dt (f32 like
 * the reference op, or bf16/f16 for the model dtype); every element is
 * written, tokens with no valid route get 0. Requires K % 32 == 0 and
 * I % 32 == 0 (tk_xpu_ext.sycl:369-370), E <= 512, top_k <= 64.
 * `workspace` holds >= sbb200_nvfp4_moe_workspace_bytes(...) device bytes,
 * not preserved between calls; concurrent calls need distinct workspaces. */
int sbb200_nvfp4_moe(void* stream, const void* hidden, const int32_t* topk_ids,
                     const float* topk_weights, const void* w13, const void* w13_scales,
                     const float* w13_global_scales, const void* w2, const void* w2_scales,
                     const float* w2_global_scales, void* workspace, size_t workspace_bytes,
                     void* out, int out_dt, size_t M, size_t E, size_t top_k, size_t K,
                     size_t I, int act_dt, int multiply_router_weight);

/* sbb200_nvfp4_moe with per-stage events, for attributing its cost (the
 * reference's nvfp4_moe_grouped_profiled_sycl + Nvfp4MoeGroupedStages,
 * src/QuixiCore-XPU/kernels/moe/nvfp4_moe/nvfp4_moe_kernel.hpp:53-83): the same
 * launches in the same order, with cudaEvent_t stage_events[i] recorded on
 * `stream` at the stage boundaries: [0] start, [1] after the route plan
 * (and the activation split), [2] after the gate/up + SwiGLU GEMM, [3] after
 * the down projection (and the split of its input), [4] after the combine.
 * n_stage_events must be SBB200_STAGE_EVENTS; NULL entries are skipped.
 * Inside a stream capture the events are recorded as external events, so
 * they stay timeable after each replay of the graph. */
#define SBB200_STAGE_EVENTS 5
int sbb200_nvfp4_moe_staged(void* stream, const void* hidden, const int32_t* topk_ids,
                            const float* topk_weights, const void* w13, const void* w13_scales,
                            const float* w13_global_scales, const void* w2, const void* w2_scales,
                            const float* w2_global_scales, void* workspace,
                            size_t workspace_bytes, void* out, int out_dt, size_t M, size_t E,
                            size_t top_k, size_t K, size_t I, int act_dt,
                            int multiply_router_weight, void* const* stage_events,
                            size_t n_stage_events);

/* Number of ids outside [-1, E) seen by the last call that used `workspace`
 * (device counter copied to the host; synchronises `stream`). The reference
 * provider rejects such ids up front (src/phase1/b70_provider.cpp:1559-1566);
 * on the device path they are dropped and counted instead. */
int sbb200_nvfp4_moe_bad_ids(void* stream, const void* workspace, uint32_t* count);

/* Device-side error word of the last call that used `workspace` (synchronises
 * `stream`): bit 0 = a pipeline wait inside a tcgen05 kernel passed its
 * deadline and the kernel abandoned its work (the result is not valid). The
 * reference's poller counts failed dispatches the same way instead of
 * hanging (src/phase7/b70_capi.h:189-193). */
int sbb200_nvfp4_moe_device_errors(void* stream, const void* workspace, uint32_t* errors);

/* Limit, in nanoseconds, of every pipeline wait inside the tcgen05 GEMM
 * kernels launched from now on (0 restores the default of 2 s); returns the
 * previous limit. A wait that runs out raises bit 0 of the device error word
 * (sbb200_nvfp4_moe_device_errors) and the kernel abandons its work and
 * returns, so the context stays usable. The limit is counted from the moment
 * the previous kernel's results are visible. Captured CUDA graphs keep the
 * limit in force at capture. Process-wide. The reference's CUDA-side wait
 * cannot time out (src/phase7/b70_capi.h:189-193); this bound replaces its
 * poller's failure counting on the device. */
uint64_t sbb200_set_kernel_wait_ns(uint64_t ns);

/* Error bits raised on the current device by any call of this library since
 * the last read, whatever workspace or stream it used (bit 0: a tcgen05 GEMM
 * wait passed its limit and that call's result is not valid). Unlike
 * sbb200_nvfp4_moe_device_errors, which sees only the last call on one
 * workspace, this keeps failures across calls and CUDA-graph replays until
 * read. Reads, clears, synchronises `stream`. No counterpart in the
 * reference (its poller counts failed dispatches, b70_capi.h:189-193). */
int sbb200_device_errors(void* stream, uint32_t* errors);

/* ---------------------------------------------------------------------------
 * Building blocks, exported for parity tests and for callers that own the
 * routing step. All stream-ordered.
 * ------------------------------------------------------------------------- */

/* W4A4 variant of sbb200_nvfp4_moe: the activations entering each GEMM
 * (hidden rows, then the SwiGLU rows) are quantised once to NVFP4 (16-element
 * e4m3 scales, vLLM ref_nvfp4_quant rounding) and multiplied with the NVFP4
 * weights by the block-scaled tensor-core MMA, fp32 accumulate.
 * Static scales (the 5090-style convention of the reference's hook, vLLM's
 * a1_gscale / a2_gscale and g1_alphas / g2_alphas, src/phase4/src/
 * shooting_brake_vllm/expert_bank.py:270-295): a13_gscale[E] and a2_gscale[E]
 * are the activation quantisation globals of each expert's inputs (scale =
 * G * blockmax / 6), and alpha13[E] / alpha2[E] multiply the MMA results
 * (alpha = 1 / (G_activation * G_weight)); the *_global_scales are unused.
 * Dynamic scales (all four NULL): each row is quantised under its own global
 * 448 * 6 / max|row| and results are scaled by 1/G_row * *_global_scales.
 * K and I multiples of 256; stage_events (NULL, or SBB200_STAGE_EVENTS
 * events) as sbb200_nvfp4_moe_staged; other arguments as sbb200_nvfp4_moe. No
 * counterpart op in the reference's extension (its W4A4 path is vLLM's). */
int sbb200_nvfp4_moe_w4a4(void* stream, const void* hidden, const int32_t* topk_ids,
                          const float* topk_weights, const void* w13, const void* w13_scales,
                          const float* w13_global_scales, const void* w2, const void* w2_scales,
                          const float* w2_global_scales, const float* a13_gscale,
                          const float* a2_gscale, const float* alpha13, const float* alpha2,
                          void* workspace, size_t workspace_bytes, void* out, int out_dt,
                          size_t M, size_t E, size_t top_k, size_t K, size_t I, int act_dt,
                          int multiply_router_weight, void* const* stage_events,
                          size_t n_stage_events);

/* Top-k routing (ops::moe_route_topk, src/QuixiCore-XPU/include/quixicore/
 * xpu/ops.hpp:262-272; moe_route.sycl.cpp:16-50): for each of M tokens pick
 * the top_k of E router logits (dt f32/f16/bf16) by k rounds of argmax with
 * the lowest index winning ties, then softmax over the chosen k. topk_ids
 * int32 [M, top_k] in selection order, topk_weights fp32 [M, top_k].
 * E <= 512, top_k <= min(E, 64). Stream-ordered. */
int sbb200_router_topk(void* stream, const void* router_logits, int dt, size_t M, size_t E,
                       size_t top_k, int32_t* topk_ids, float* topk_weights);

/* sbb200_nvfp4_moe with the routing computed in front of the permute from
 * router_logits [M, E] (logits_dt): the top-k ids and softmax weights are
 * written to topk_ids / topk_weights (outputs here) and used by the forward.
 * Up to 4096 routes the routing runs inside the route-plan kernel itself, so
 * it adds no launch. Same workspace as sbb200_nvfp4_moe. */
int sbb200_nvfp4_moe_from_logits(void* stream, const void* hidden, const void* router_logits,
                                 int logits_dt, int32_t* topk_ids, float* topk_weights,
                                 const void* w13, const void* w13_scales,
                                 const float* w13_global_scales, const void* w2,
                                 const void* w2_scales, const float* w2_global_scales,
                                 void* workspace, size_t workspace_bytes, void* out, int out_dt,
                                 size_t M, size_t E, size_t top_k, size_t K, size_t I,
                                 int act_dt, int multiply_router_weight);

/* Stable route permutation (nvfp4_moe_grouped.sycl.cpp:140-204 with the CPU
 * tier's order, src/phase7/cpu_expert_capi.cpp:563-599): counts int32 [E],
 * offsets int32 [E + 1], sorted int32 [M*top_k] (route ids r = m*top_k + k
 * grouped by expert, r ascending within an expert; entries past offsets[E]
 * are left untouched), slot_of int32 [M*top_k] (-1 for dropped ids).
 * `scratch` needs sbb200_route_plan_scratch_bytes(M*top_k, E) bytes;
 * `bad_ids` (uint32, may be NULL) is incremented by the count of ids outside
 * [-1, E). */
size_t sbb200_route_plan_scratch_bytes(size_t routes, size_t E);
int sbb200_route_plan(void* stream, const int32_t* topk_ids, size_t M, size_t top_k, size_t E,
                      int32_t* counts, int32_t* offsets, int32_t* sorted, int32_t* slot_of,
                      void* scratch, uint32_t* bad_ids);

/* sbb200_route_plan without allocation, for callers that cannot give the
 * library device memory: serving engines whose device memory is owned by a
 * pooling allocator sized before the model runs, and FFI bindings (ctypes,
 * cgo, JNI) that hold only the tensors they were handed and have no device
 * allocator. Same arguments and results as sbb200_route_plan minus the
 * scratch: its scratch is a fixed 128 KB array in the library's device image
 * (held on every device that loads the library until exit), so it handles at
 * most 262144 routes (M * top_k) and E <= 512; larger calls fail with
 * SBB200_EUNSUPPORTED. Nothing is allocated by any call. The first call on a
 * device resolves that array's device address (cudaGetSymbolAddress), so make
 * the first call on each device before any stream capture; the address is
 * kept for the life of the process, so the entry point is not usable on a
 * device after cudaDeviceReset. All calls share the array and each call
 * overwrites what the previous one left there: calls that overlap on the GPU
 * (different streams, or several host threads) race and must be serialised
 * by the caller. Has no counterpart in the reference. */
int sbb200_route_plan_static(void* stream, const int32_t* topk_ids, size_t M, size_t top_k,
                             size_t E, int32_t* counts, int32_t* offsets, int32_t* sorted,
                             int32_t* slot_of, uint32_t* bad_ids);

/* Bit-exact NVFP4 dequant: out[r, c] = e2m1 * fp32(e4m3(sf[r, c/16]) * g[r /
 * rows_per_scale]) (src/phase7/cpu_expert_capi.cpp:301-346). q [rows, cols/2],
 * sf [rows, cols/16], out fp32 [rows, cols]; cols % 16 == 0. */
int sbb200_nvfp4_dequant(void* stream, const void* q, const void* sf, const float* g,
                         size_t rows_per_scale, float* out, size_t rows, size_t cols);

/* NVFP4 quantiser with vLLM ref_nvfp4_quant semantics (the quantiser of the
 * reference's fixtures, src/phase7/nvfp4_testutil.py): x [rows, cols] in
 * in_dt, quantisation global gq[r / rows_per_scale] (= 448*6/amax); writes
 * q [rows, cols/2] and sf [rows, cols/16]. */
int sbb200_nvfp4_quantize(void* stream, const void* x, int in_dt, const float* gq,
                          size_t rows_per_scale, void* q, void* sf, size_t rows, size_t cols);

/* ---------------------------------------------------------------------------
 * Provider: registered layers and an owned workspace, the device-resident
 * replacement of the reference's B70 provider C-ABI (src/phase7/b70_capi.h:
 * 44-321, src/phase1/b70_provider.hpp:86-230) without the doorbell/poller
 * transport. Weights stay caller-owned device memory.
 * ------------------------------------------------------------------------- */

typedef struct sbb200_provider sbb200_provider_t;

/* 48-byte POD, field for field the reference's sb_b70_health_t
 * (src/phase7/b70_capi.h:28-41); its `reserved` word carries the device error
 * word of the provider's last forward here (bit 0: a kernel wait passed its
 * limit and that forward's result is not valid; bit 31: the word could not
 * be read). */
typedef struct sbb200_health {
  uint64_t generation;
  uint64_t dispatches;
  uint64_t allocations;
  uint64_t last_error_bytes;
  uint32_t loaded;
  uint32_t pending;
  uint32_t stopped;
  uint32_t device_errors;
} sbb200_health_t;

/* Create a provider on `device` able to serve batches up to max_tokens tokens
 * of top_k routes for layers of at most max_E experts, hidden K and
 * intermediate I. Allocates its workspace once. NULL on failure. */
sbb200_provider_t* sbb200_create(int device, size_t max_tokens, size_t top_k, size_t max_E,
                                 size_t K, size_t I);
void sbb200_destroy(sbb200_provider_t* p);

/* Register layer `layer`'s device weights (pointers are kept, not copied). */
int sbb200_register_layer(sbb200_provider_t* p, size_t layer, size_t E, const void* w13,
                          const void* w13_scales, const float* w13_global_scales,
                          const void* w2, const void* w2_scales,
                          const float* w2_global_scales);

/* Routed-expert forward of a registered layer on `stream` (the issue step of
 * src/phase1/b70_provider.cpp:1530-1849 without the host copies). M must be
 * <= max_tokens; ids outside [-1, E) are dropped and counted in health. */
int sbb200_moe_forward(sbb200_provider_t* p, size_t layer, void* stream, const void* hidden,
                       int act_dt, const int32_t* topk_ids, const float* topk_weights,
                       void* out, int out_dt, size_t M, int multiply_router_weight);

/* Health snapshot + last error copy-out (src/phase7/b70_capi.h:159-172):
 * 0 ok, -1 invalid arguments, -2 buffer too small (truncated copy written,
 * last_error_bytes holds the size needed). After a forward it synchronises
 * the provider's device to read device_errors, so it is not to be called
 * inside a stream capture. */
int sbb200_health(sbb200_provider_t* p, sbb200_health_t* health, char* last_error,
                  size_t last_error_size);

/* ---------------------------------------------------------------------------
 * SBEXP001 expert bank (the reference's on-disk NVFP4 bank: writer
 * src/phase1/extract_experts.py:51-128, 234-281; C++ reader
 * src/phase1/b70_provider.cpp:194-246, 866-934). Opened read-only by mmap and
 * validated like the reference (magic, reserved field, geometry, file size);
 * the INT4 bank (SBINT401) is not part of this path and is rejected.
 * ------------------------------------------------------------------------- */

typedef struct sbb200_bank sbb200_bank_t;

/* NULL on failure (sbb200_last_error says why). */
sbb200_bank_t* sbb200_bank_open(const char* path);

int sbb200_bank_info(sbb200_bank_t* bank, size_t* layers, size_t* experts, size_t* hidden,
                     size_t* intermediate);

/* One expert's planes into HOST buffers (any pointer may be NULL to skip):
 * w13 [2I, H/2] (gate rows then up rows), w13_scales [2I, H/16], w2 [H, I/2],
 * w2_scales [H, I/16], and the two fp32 dequant multipliers. */
int sbb200_bank_read_expert(sbb200_bank_t* bank, size_t layer, size_t expert, void* w13,
                            void* w13_scales, float* w13_global_scale, void* w2,
                            void* w2_scales, float* w2_global_scale);

/* Experts [expert_begin, expert_begin + expert_count) of `layer` into DEVICE
 * planes in the layout of sbb200_nvfp4_moe (row i = expert expert_begin + i):
 * w13 [n, 2I, H/2], w13_scales [n, 2I, H/16], w13_global_scales fp32 [n], w2
 * [n, H, I/2], w2_scales [n, H, I/16], w2_global_scales fp32 [n]. Copies on
 * `stream` through pinned staging and returns when they are complete. */
int sbb200_bank_load(sbb200_bank_t* bank, void* stream, size_t layer, size_t expert_begin,
                     size_t expert_count, void* w13, void* w13_scales,
                     float* w13_global_scales, void* w2, void* w2_scales,
                     float* w2_global_scales);

void sbb200_bank_close(sbb200_bank_t* bank);

/* ---------------------------------------------------------------------------
 * Expert parallelism over NVLink: one process per GPU of one node, the E
 * routed experts sharded contiguously (the first E % world ranks hold one
 * extra), tokens kept by the rank that owns them. Replaces the reference's
 * multi-card split, where every card sees all routes with foreign experts as
 * -1 and the host sums the per-card outputs (src/phase4/src/
 * shooting_brake_vllm/routed_experts.py:354-382, 2460-2463, 2522-2524).
 * Bring-up: create on every rank, exchange the SBB200_EP_HANDLE_BYTES handle
 * of each rank (any host transport; rank order), connect. Every rank then
 * calls sbb200_ep_forward once per step, in the same order; the exchange is
 * device-resident (no NCCL on the data path, no host synchronisation).
 * ------------------------------------------------------------------------- */

#define SBB200_EP_HANDLE_BYTES 64

typedef struct sbb200_ep sbb200_ep_t;

/* Expert shard [*begin, *begin + *count) of `rank`. */
int sbb200_ep_shard(size_t E, int world, int rank, size_t* begin, size_t* count);

/* Exchange state of `rank` of `world` on `device` for up to max_tokens
 * tokens per rank (hidden K in act_dt, top_k routes, E experts in total,
 * intermediate I; K and I multiples of 256). w4a4 != 0 runs each shard's
 * experts as sbb200_nvfp4_moe_w4a4 with dynamic per-row scales. NULL on
 * failure. */
sbb200_ep_t* sbb200_ep_create(int device, int rank, int world, size_t max_tokens, size_t top_k,
                              size_t E, size_t K, size_t I, int act_dt, int w4a4);

/* This rank's exchange-buffer handle (SBB200_EP_HANDLE_BYTES bytes). */
int sbb200_ep_ipc_handle(sbb200_ep_t* ep, void* out, size_t size);

/* Map every other rank's buffer: `handles` holds world handles in rank order. */
int sbb200_ep_connect(sbb200_ep_t* ep, const void* handles, size_t size);

/* One expert-parallel layer step on `stream`: this rank's M tokens (hidden
 * [M, K] in act_dt, topk_ids int32 [M, top_k] with global expert ids,
 * topk_weights fp32 [M, top_k]) in, out [M, K] in out_dt; w13..w2_global_scales
 * are this rank's shard (sbb200_ep_shard) in the layout of sbb200_nvfp4_moe,
 * indexed by local expert id. M may be 0 (the rank still serves its experts).
 * Each route's expert output is computed on the rank that holds the expert
 * and summed on the token's own rank in ascending k with the router weights,
 * the arithmetic of sbb200_nvfp4_moe's combine. */
int sbb200_ep_forward(sbb200_ep_t* ep, void* stream, const void* hidden, const int32_t* topk_ids,
                      const float* topk_weights, size_t M, const void* w13,
                      const void* w13_scales, const float* w13_global_scales, const void* w2,
                      const void* w2_scales, const float* w2_global_scales, void* out,
                      int out_dt, int multiply_router_weight);

/* sbb200_ep_forward that also records SBB200_EP_STAGE_EVENTS cudaEvent_t on
 * `stream`: [0] start, [1] after publish, [2] after the gather (including the
 * wait for every rank's publish), [3] after the route plan and the pulled
 * activation split, [4] after gate/up, [5] after down (which pushes each
 * route's row to its source), [6] = [5], [7] after the final sum (including
 * the wait for every rank). In decode-sized steps (world * max_tokens *
 * top_k <= 1024) the activation split does the publish and the gather
 * itself, so [0] = [1] = [2]. No counterpart in the reference; it times the
 * exchange against the GEMMs. */
#define SBB200_EP_STAGE_EVENTS 8
int sbb200_ep_forward_staged(sbb200_ep_t* ep, void* stream, const void* hidden,
                             const int32_t* topk_ids, const float* topk_weights, size_t M,
                             const void* w13, const void* w13_scales,
                             const float* w13_global_scales, const void* w2,
                             const void* w2_scales, const float* w2_global_scales, void* out,
                             int out_dt, int multiply_router_weight, void* const* stage_events,
                             size_t n_stage_events);

/* Error bits raised on the device since the last read (bit 0: a wait for
 * another rank passed its 2 s deadline); reads, clears, synchronises. */
int sbb200_ep_device_errors(sbb200_ep_t* ep, void* stream, uint32_t* errors);

/* Number of kernels one sbb200_ep_forward step launches on its stream, or
 * -1 for a null handle: 5 for decode-sized steps (exchange split, gate/up,
 * SwiGLU split, down, final sum), more for larger ones (publish, gather and
 * the route plan run as kernels of their own). No counterpart in the
 * reference. */
int sbb200_ep_launches(const sbb200_ep_t* ep);

void sbb200_ep_destroy(sbb200_ep_t* ep);

#ifdef __cplusplus
}
#endif

#endif /* SBB200_H */
