// Shared device helpers and host-side error / table machinery of libcorm_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <cstdlib>
#include <utility>
#include <string>

#include "cormorant_b200.h"

namespace corm {

// ---------------------------------------------------------------- errors (host)
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_status(const char* where);  // CORM_OK or CORM_ECUDA after a launch
int check_device();                  // CORM_OK when the current device is sm_100

// Per-device scratch owned by the library (grow-only; used when a job passes
// no workspace).  Returns nullptr on failure (error set).
void* scratch(size_t bytes, cudaStream_t stream);

// ---------------------------------------------------------------- tables
// Device copies of the unit tables, uploaded once per device on first use.
struct DeviceTables {
  const int16_t* act[7];     // 65536-entry activation tables (index raw + 32768); [3] unused
  const int32_t* smx_tab;    // 4096-entry softmax TAB
  uint64_t* ro_sig;          // 4096 sigmoid entries {D << 25 | T} (OP_TLOAD words)
  uint32_t* ro_rsq;          // 8192 rsqrt entries
};
const DeviceTables* tables();  // nullptr on failure (error set)

// Kernel-level tracing: every launch site holds a ProfScope, which counts the
// launch and, while profiling is enabled (corm_profile_enable), brackets it
// with CUDA events on the launching stream.
struct ProfScope {
  ProfScope(const char* name, cudaStream_t stream);
  ~ProfScope();
  const char* name;
  cudaStream_t stream;
  int slot;
};

// Host table builders (tables.cpp): bit-exact restatements of the reference's
// vectorop_act.kernel_table, vectorop_smx.TAB and rowops_spec tables.
void build_act_table(int act, uint32_t alpha, int16_t* out);
void build_smx_tab(int32_t* out);
void build_rowops_image(uint8_t* out65536);

}  // namespace corm

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ int64_t corm_sat16(int64_t v) {
  return v > 32767 ? 32767 : (v < -32768 ? -32768 : v);
}
__device__ __forceinline__ int64_t corm_sat32(int64_t v) {
  return v > 2147483647LL ? 2147483647LL : (v < -2147483648LL ? -2147483648LL : v);
}
__device__ __forceinline__ int64_t corm_wrap32(int64_t v) { return (int64_t)(int32_t)(uint32_t)(uint64_t)v; }

// round half to even of x / 2^k (k >= 0), 128-bit
__device__ __forceinline__ __int128 corm_rne_shr128(__int128 x, int k) {
  if (k <= 0) return x << (-k);
  __int128 q = x >> k;
  __int128 r = x - (q << k);
  __int128 half = (__int128)1 << (k - 1);
  return q + ((r > half || (r == half && (q & 1))) ? 1 : 0);
}
__device__ __forceinline__ int64_t corm_rne_shr64(int64_t x, int k) {
  if (k <= 0) return x << (-k);
  int64_t q = x >> k;
  int64_t r = x - (q << k);
  int64_t half = (int64_t)1 << (k - 1);
  return q + ((r > half || (r == half && (q & 1))) ? 1 : 0);
}
// the same for |x| < 2^62, 0 <= k <= 63, without the remainder: adding
// 2^(k-1) - 1 plus the parity of floor(x / 2^k) carries into the quotient
// exactly when the remainder is above half, or equal to it with an odd quotient
__device__ __forceinline__ int64_t corm_rne_shr64f(int64_t x, int k) {
  if (k == 0) return x;
  return (x + ((int64_t)1 << (k - 1)) - 1 + ((x >> k) & 1)) >> k;
}
__device__ __forceinline__ int64_t corm_sat16_128(__int128 x) {
  return x > 32767 ? 32767 : (x < -32768 ? -32768 : (int64_t)x);
}
__device__ __forceinline__ int64_t corm_sat32_128(__int128 x) {
  return x > 2147483647 ? 2147483647 : (x < -(__int128)2147483648LL ? -2147483648LL : (int64_t)x);
}

static inline unsigned corm_blocks(size_t work, unsigned per_block, unsigned cap = 148u * 32u) {
  size_t b = (work + per_block - 1) / per_block;
  if (b < 1) b = 1;
  return (unsigned)(b > cap ? cap : b);
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with corm_launch_pdl may start while the kernel before it
// on the stream is still running: it must call corm_pdl_wait() before its first
// global-memory access (the wait returns once the previous grid has completed
// and its writes are visible), and calls corm_pdl_trigger() to let the next
// kernel launch early in turn.  Only the launch latency and the prologue
// overlap; every read and write stays ordered after the previous kernel.
__device__ __forceinline__ void corm_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void corm_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// CORM_NO_PDL=1: plain launches (for comparisons)
static inline bool corm_pdl_enabled() {
  const char* e = getenv("CORM_NO_PDL");
  return !(e && e[0] == '1');
}

template <typename... KArgs, typename... Args>
static inline cudaError_t corm_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                          cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = corm_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
