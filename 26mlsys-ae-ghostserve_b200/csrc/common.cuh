// common.cuh — shared helpers of libgsec: error reporting, 16-byte vector
// access, launch sizing and GF(2^8)/GF(2^16) arithmetic.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/gsec.h"

namespace gsec {

// ---------------------------------------------------------------- errors ----

void set_error(const char* fmt, ...);
const char* last_error();

#define GSEC_REQUIRE(cond, ...)               \
  do {                                        \
    if (!(cond)) {                            \
      ::gsec::set_error(__VA_ARGS__);         \
      return GSEC_EINVAL;                     \
    }                                         \
  } while (0)

// Returns GSEC_ECUDA with the launch error if the last launch failed.
int check_launch(const char* what);
// GSEC_OK, or GSEC_ECUDA with the message of `rc` (a cudaLaunchKernelEx result).
int launch_rc(cudaError_t rc, const char* what);

inline cudaStream_t as_stream(gsec_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#ifndef GSEC_PDL
#define GSEC_PDL 1
#endif
// Programmatic dependent launch: a kernel launched with launch_pdl may be
// started while the previous kernel in its stream is still finishing. Its CTAs
// set up (shared-memory barriers, tables) and then wait in grid_dep_wait()
// until every prerequisite grid has completed and its memory operations are
// visible, so no global memory is touched early; grid_dep_launch() lets the
// next kernel in the stream be scheduled the same way. Back-to-back launches
// then overlap their launch latency and ramp-up with the previous one's tail.
// Kernels launched without the attribute pass through both instructions.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = GSEC_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#ifndef GSEC_BALANCED_GRID
#define GSEC_BALANCED_GRID 1
#endif
// Grid for `items` equal work items handed out round-robin (item it to CTA
// it % grid), at most `max_grid` CTAs: the fewest CTAs that still finish in
// the same number of rounds, so every CTA gets either ceil(items / grid) or
// one item fewer, and no last round runs with a fraction of the CTAs while
// the rest sit idle (5464 items on 740 resident CTAs: 683 CTAs x 8 items).
inline int64_t balanced_grid(int64_t items, int64_t max_grid) {
  if (items < 1) return 1;
  if (max_grid < 1) max_grid = 1;
  if (items <= max_grid) return items;
  if (!GSEC_BALANCED_GRID) return max_grid;
  const int64_t rounds = (items + max_grid - 1) / max_grid;
  return (items + rounds - 1) / rounds;
}

// Per-device cache of kernels' launch shapes: a kernel's dynamic shared
// memory attribute is raised once and its resident-CTA count is queried once
// per (device, kernel, shared-memory size), instead of on every launch.
int current_device();

class LaunchCache {
 public:
  template <typename K>
  int blocks_per_sm(K kernel, int threads, size_t dyn_smem) {
    const void* fn = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lock(mu_);
    const int dev = current_device();
    if (dev < 0) return -1;
    size_t& attr = attr_[{dev, fn}];
    if (dyn_smem > attr) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_smem) != cudaSuccess)
        return -1;
      attr = dyn_smem;
    }
    const Key key{dev, fn, dyn_smem, threads};
    auto it = per_sm_.find(key);
    if (it != per_sm_.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, dyn_smem) != cudaSuccess) return -1;
    if (n < 1) n = 1;
    per_sm_[key] = n;
    return n;
  }

 private:
  struct Key {
    int dev;
    const void* fn;
    size_t smem;
    int threads;
    bool operator<(const Key& o) const {
      if (dev != o.dev) return dev < o.dev;
      if (fn != o.fn) return fn < o.fn;
      if (smem != o.smem) return smem < o.smem;
      return threads < o.threads;
    }
  };
  std::mutex mu_;
  std::map<std::pair<int, const void*>, size_t> attr_;
  std::map<Key, int> per_sm_;
};

// The process-wide cache.
LaunchCache& launch_cache();

// Division of 32-bit values by a run-time constant d (1 <= d < 2^32), with the
// multiplier precomputed on the host (Granlund-Montgomery, round-up variant):
// s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1, q = (umulhi(x, m) + x) >> s.
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    while ((1ull << s) < div) ++s;
    m = (uint32_t)(((((1ull << s) - div) << 32) / div) + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t x) const {
    return (uint32_t)((((uint64_t)__umulhi(x, m)) + x) >> s);
  }
};

// ---------------------------------------------------------- vector access ---

__device__ __forceinline__ uint4 vxor(uint4 a, uint4 b) {
  return make_uint4(a.x ^ b.x, a.y ^ b.y, a.z ^ b.z, a.w ^ b.w);
}

__device__ __forceinline__ uint4 vzero() { return make_uint4(0u, 0u, 0u, 0u); }

// 16 bytes starting at any byte address p, assembled from the aligned 16-byte
// block(s) that hold them: one block when p is aligned, else two, both of which
// contain bytes of [p, p + 16) (so nothing outside the aligned span of the
// requested bytes is read). Plain cached loads: a neighbouring thread reads the
// same blocks.
__device__ __forceinline__ uint4 ldu16(const void* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t m = (uint32_t)(a & 15u);
  const uint4* q = reinterpret_cast<const uint4*>(a - m);
  const uint4 lo = q[0];
  if (m == 0) return lo;
  const uint4 hi = q[1];
  const uint32_t e[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  const uint32_t sh = (m & 3u) * 8u;
  uint32_t o[4];
  switch (m >> 2) {  // whole words of the shift; the byte part is a funnel shift
    case 0:
#pragma unroll
      for (int l = 0; l < 4; ++l) o[l] = __funnelshift_r(e[l], e[l + 1], sh);
      break;
    case 1:
#pragma unroll
      for (int l = 0; l < 4; ++l) o[l] = __funnelshift_r(e[l + 1], e[l + 2], sh);
      break;
    case 2:
#pragma unroll
      for (int l = 0; l < 4; ++l) o[l] = __funnelshift_r(e[l + 2], e[l + 3], sh);
      break;
    default:
#pragma unroll
      for (int l = 0; l < 4; ++l) o[l] = __funnelshift_r(e[l + 3], e[l + 4], sh);
      break;
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ------------------------------------------------------------- GF(2^8) ------
// Field GF(2)[x]/(x^8+x^4+x^3+x^2+1) (0x11d), generator x (= 2).

__host__ __device__ __forceinline__ uint32_t gf8_mul(uint32_t a, uint32_t b) {
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (b & 1u) r ^= a;
    b >>= 1;
    a <<= 1;
    if (a & 0x100u) a ^= 0x11du;
  }
  return r & 0xffu;
}

// ------------------------------------------------------------ GF(2^16) ------
// Field GF(2)[x]/(x^16+x^12+x^3+x+1) (0x1100B), generator x, as built by the
// reference's init_gf_tables (benchmark/rs/main.py:39-54).

__host__ __device__ __forceinline__ uint32_t gf16_mul(uint32_t a, uint32_t b) {
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (b & 1u) r ^= a;
    b >>= 1;
    a <<= 1;
    if (a & 0x10000u) a ^= 0x1100bu;
  }
  return r & 0xffffu;
}

// Host-side tables and inverses (defined in gf.cpp part of api.cu).
uint8_t gf8_inv(uint8_t a);
uint16_t gf16_exp(int e);          // alpha^e, e in [0, 2*65535)
uint16_t gf16_log(uint16_t a);     // discrete log, a != 0
uint16_t gf16_mul_tab(uint16_t a, uint16_t b);  // exp/log multiply (reference form)
uint16_t gf16_div_tab(uint16_t a, uint16_t b);

// Maximum shard pointers a kernel takes by value.
constexpr int kMaxShards = 34;

}  // namespace gsec
