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

}  // namespace nb
