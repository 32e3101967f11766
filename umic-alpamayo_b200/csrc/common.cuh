// Shared helpers for the umic_b200 kernels: bf16 vector packing, cache-hinted
// loads, host-side argument checks and the per-thread error message.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <mutex>
#include <cstdio>

#include "../../include/umic_b200.h"

namespace umic {

// ---------------------------------------------------------------- host side

// Records a one-line reason and returns `code` (thread-local message buffer).
int fail(int code, const char* fmt, ...);
void clear_error();

// Device-side error word of the current device (allocated by the runtime as a
// __device__ symbol; its address is resolved once per device).
uint32_t* device_error_word();

// Streaming multiprocessor count of the current device (cached per device).
int sm_count();

// Test hook of the bounded-wait abort path (umic_debug_stall): true, with the armed wait
// limit in *limit, exactly once after `kernel` was armed; false otherwise.
constexpr int kStallGemm = 1;
constexpr int kStallGemv = 2;
constexpr int kGemvGeneralMerge = 3;  // not a stall: the next GEMV skips its fast merge
bool take_stall(int kernel, long long* limit);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Asks (once per device) for the largest shared-memory carveout for `Kernel`. The
// small streaming kernels that precede a streaming GEMV then leave their SMs
// configured so the GEMV's CTAs (about 193 KB of shared memory) can become
// resident beside them as soon as they allow the dependent launch.
template <auto Kernel>
inline void prefer_max_shared() {
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [] {
    cudaFuncSetAttribute(Kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    cudaGetLastError();  // a refusal only costs the overlap
  });
}

// Launches `kernel` with programmatic stream serialization: its CTAs may become
// resident while the previous kernel of the stream finishes (once that kernel has
// called griddepcontrol.launch_dependents), so the launch latency hides behind its
// tail. The kernel must call wait_prerequisite() before it reads anything the previous
// kernel writes (or writes anything that kernel reads).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Maps the launch status to UMIC_ERR_LAUNCH with the CUDA error string (a failed
// cudaLaunchKernelEx is reported here too: it sets the runtime's last error).
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UMIC_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return UMIC_OK;
}

// -------------------------------------------------------------- device side

// Lets the next kernel in the stream begin launching now if it was launched with
// programmatic stream serialization (the streaming GEMV is). That kernel still
// waits for this grid to complete (griddepcontrol.wait) before it reads anything
// this grid writes; without such a dependent this is a no-op.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Waits until the previous kernel of the stream has completed and its writes are
// visible (a no-op unless this grid was launched with launch_pdl).
__device__ __forceinline__ void wait_prerequisite() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Eight bf16 values travel as one 16-byte vector.
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 is the high half of an fp32: shifting is the exact conversion.
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return v;
}

// Read-once data: bypass L1 allocation so it does not evict reused lines.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Reused read-only data (weights of a norm, cos/sin tables, GEMV activations).
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void st_vec(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// Loads 8 consecutive weights as fp32 from a bf16 or fp32 array.
__device__ __forceinline__ void load_w8(const void* w, int dtype, int64_t idx, float (&f)[8]) {
  if (dtype == UMIC_DTYPE_FP32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(w) + idx);
    float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8(ld_cached(static_cast<const __nv_bfloat16*>(w) + idx), f);
  }
}

__device__ __forceinline__ float load_w1(const void* w, int dtype, int64_t idx) {
  if (dtype == UMIC_DTYPE_FP32) return __ldg(static_cast<const float*>(w) + idx);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[idx]);
}

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace umic
