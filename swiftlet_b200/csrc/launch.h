// Kernel launch helper: cudaLaunchKernelEx with optional programmatic
// dependent launch; the launch status is checked directly (never through
// cudaGetLastError, which can hold an older, unrelated error).
#pragma once

#include <string>
#include <vector>

#include "common.h"

namespace swl {

// While set, every launcher on this thread appends the kernel family it
// chose ("igemv", "idown", "delta", ...), so a test can assert which kernels a
// decode step runs (the tensor-core, slice or register-streaming ones).
extern thread_local std::vector<std::string>* g_path_log;
inline void path_note(const char* family) {
  if (g_path_log) g_path_log->push_back(family);
}

template <typename Kern, typename... Args>
void launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (smem > 48 * 1024) SWL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  SWL_CUDA(cudaLaunchKernelEx(&cfg, k, args...));
}

// The same with thread-block clusters of `cluster` CTAs (grid divisible by it).
template <typename Kern, typename... Args>
void launch_cluster(Kern k, dim3 grid, dim3 block, dim3 cluster, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (smem > 48 * 1024) SWL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  SWL_CUDA(cudaLaunchKernelEx(&cfg, k, args...));
}

}  // namespace swl
