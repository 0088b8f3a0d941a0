// Shared device helpers for the cwen B200 kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#define CW_DEV __device__ __forceinline__
#define CW_HOST_DEV __host__ __device__ __forceinline__

namespace cw {

// Programmatic dependent launch (PDL).  Every decode-step kernel is launched
// with programmatic stream serialization: it may start while the previous
// kernel of the stream still runs.  Each kernel therefore calls pdl_wait()
// before it touches any memory an earlier kernel writes or reads (the wait
// returns once the previous grid has completed and its writes are visible;
// that grid itself waited on its predecessor, so the chain is ordered), and
// calls pdl_trigger() early so that its successor's launch overlaps its run.
CW_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CW_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with a thread-block cluster of cl CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      int cl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cl;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Largest cluster size in {8, 4, 2, 1} that divides n.
inline int cluster_split(int n) { return n % 8 == 0 ? 8 : (n % 4 == 0 ? 4 : (n % 2 == 0 ? 2 : 1)); }

// Return the error of a launch from a launcher that returns cudaError_t.
#define CW_TRY(expr)                  \
  do {                                \
    cudaError_t _e = (expr);          \
    if (_e != cudaSuccess) return _e; \
  } while (0)

// Prefer the largest shared-memory carveout for a kernel.  With every kernel
// of the decode step on the same carveout, an SM never reconfigures its
// L1/shared split between consecutive kernels (measured ~1.5 us per switch).
template <class F>
inline cudaError_t carveout_max(F *fn) {
  return cudaFuncSetAttribute(reinterpret_cast<const void *>(fn), cudaFuncAttributePreferredSharedMemoryCarveout,
                              (int)cudaSharedmemCarveoutMaxShared);
}

CW_DEV uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// lop3 with an immediate truth table.
template <int LUT>
CW_DEV uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
CW_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1, const float (&c)[4]) {
  asm(  // no side effects: the compiler may schedule it freely
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

CW_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
CW_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace cw
