// Shared-memory opt-in for kernels launched with more than 48 KB of dynamic
// shared memory. The attribute is set once per (kernel, device) so that no
// attribute call happens while a decode step is being captured into a graph.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

namespace nb {

inline cudaError_t allow_smem(const void* kern, size_t smem) {
  if (smem == 0) return cudaSuccess;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(kern, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= smem) return cudaSuccess;
  // Opt in to the B200 per-block maximum (227 KB, static shared memory
  // included) once; later launches need no call.
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  if (smem + fa.sharedSizeBytes <= 48 * 1024) {
    done[key] = smem;
    return cudaSuccess;
  }
  const size_t want = 227 * 1024 - fa.sharedSizeBytes;
  if (smem > want) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
  if (e == cudaSuccess) done[key] = want;
  return e;
}

// Launch with programmatic stream serialization: the kernel may begin while
// the previous kernel in the stream finishes; it must call pdl_wait() before
// touching anything that kernel reads or writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace nb
