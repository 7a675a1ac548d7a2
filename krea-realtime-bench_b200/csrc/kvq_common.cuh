// Internal helpers shared by the kvq CUDA sources: error state, group layouts,
// bf16 bit tricks. Device code targets sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "kvq.h"

namespace kvq {

// ---------------------------------------------------------------- error state
// Thread-local message of the last failing call (kvq_last_error()).
void set_error(const char* fmt, ...);
void clear_error();

#define KVQ_REQUIRE(cond, code, ...)   \
  do {                                 \
    if (!(cond)) {                     \
      ::kvq::set_error(__VA_ARGS__);   \
      return (code);                   \
    }                                  \
  } while (0)

// Returns KVQ_OK, or KVQ_ERR_CUDA with the message of a pending launch error.
int check_launch(const char* what);

// KVQ_ERR_DEVICE unless the current device is compute capability 10.x.
int require_sm100();

// ---------------------------------------------------------------- group layouts
// The channel-group maps the reference uses (quant_kv.py:62-82), head_dim 128.
// Each is a run of contiguous groups given by its G+1 edges.
enum LayoutId : int {
  kLayoutGeneric = 0,
  kLayoutBands = 1,    // G=3  [0,44) [44,86) [86,128)
  kLayoutBands2 = 2,   // G=6
  kLayoutBands4 = 3,   // G=12
  kLayoutBlind32 = 4,  // G=4
  kLayoutBlind64 = 5,  // G=2
};

struct LayoutBands {
  static constexpr int G = 3;
  static constexpr int E[G + 1] = {0, 44, 86, 128};
};
struct LayoutBands2 {
  static constexpr int G = 6;
  static constexpr int E[G + 1] = {0, 22, 44, 66, 86, 108, 128};
};
struct LayoutBands4 {
  static constexpr int G = 12;
  static constexpr int E[G + 1] = {0, 12, 24, 36, 44, 56, 68, 80, 86, 98, 110, 122, 128};
};
struct LayoutBlind32 {
  static constexpr int G = 4;
  static constexpr int E[G + 1] = {0, 32, 64, 96, 128};
};
struct LayoutBlind64 {
  static constexpr int G = 2;
  static constexpr int E[G + 1] = {0, 64, 128};
};

// Largest head_dim / group count the generic kernels accept.
constexpr int kMaxHeadDim = 256;
constexpr int kMaxGroups = 256;

// Validated group map, passed to kernels by value.
struct GroupMap {
  uint8_t gid[kMaxHeadDim];  // group of each channel
};

// Validates chan_band (host int32[D], values in [0,G), every group non-empty)
// and returns the specialised layout it matches, or kLayoutGeneric. On error
// returns a negative status with the message set.
int resolve_layout(const int32_t* chan_band, int head_dim, int n_groups, GroupMap* map);

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
// float -> bf16 bits, round to nearest even (cvt.rn.bf16.f32).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
}
// Two floats -> packed bf16x2 (lo in bits 0..15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Programmatic dependent launch. pdl_wait(): no global memory access of this
// grid may come before the grid ahead of it on the stream has completed and its
// writes are visible (a no-op when that grid was not launched as a programmatic
// prerequisite). pdl_launch_dependents(): the next grid on the stream may be
// scheduled once every CTA of this one has executed it (it still waits for this
// grid's completion in its own pdl_wait()), so its launch overlaps this grid's
// tail instead of following it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with the programmatic-stream-serialization attribute (the kernel must
// call pdl_wait() before its first global memory access).
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_global_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

}  // namespace kvq
