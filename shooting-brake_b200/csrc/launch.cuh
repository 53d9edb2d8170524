// Kernel launches with programmatic dependent launch (PDL).
//
// A kernel launched with pdl = true may start while the previous kernel on
// the stream is still draining: its CTAs run their local prologue (shared
// memory and mbarrier set-up, tensor-memory allocation, tensor-map prefetch)
// and then block in pdl_wait() until that kernel has completed and its
// writes are visible. That hides the launch gap between the dependent
// kernels of one forward. The first kernel of a call is launched with
// pdl = false, so nothing overlaps work from before the call.
#pragma once

#include <cuda_runtime.h>

namespace sbb {

// Blocks until the preceding kernel in the stream has completed and flushed
// (returns at once for a kernel launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next PDL kernel in the stream launch before this one ends.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Records a stage event on `stream`; inside a stream capture as an external
// event node, so the event stays timeable after each replay of the graph
// (outside a capture a plain record, the only form allowed there).
inline cudaError_t record_stage_event(cudaEvent_t ev, cudaStream_t stream) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  const cudaError_t err = cudaStreamIsCapturing(stream, &st);
  if (err != cudaSuccess) return err;
  return st == cudaStreamCaptureStatusActive
             ? cudaEventRecordWithFlags(ev, stream, cudaEventRecordExternal)
             : cudaEventRecord(ev, stream);
}

}  // namespace sbb
