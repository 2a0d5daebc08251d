// pipe.cuh — a TMA bulk-copy staging ring for streaming kernels.
//
// One producer lane issues cp.async.bulk copies (global -> shared, no
// multicast) of the next stage's input cells and signals a "full" mbarrier via
// its transaction count; the consumer threads wait on it, compute from shared
// memory and arrive on the stage's "empty" mbarrier so the producer may refill
// it.  Many stages in flight per SM keep tens of KB of loads outstanding with
// no register cost, which is what an HBM-bound XOR/GF kernel needs on B200.
//
// Every wait is bounded (kWaitNs of %globaltimer).  A wait that gives up sets
// a bit in the translation unit's device status word and the thread returns;
// a producer that gives up first waits (again bounded) for the copies it has
// in flight, so no bulk copy lands in shared memory after its CTA has exited.
#pragma once

#include <stdint.h>

namespace gsec {
namespace pipe {

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t* b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the phase of parity `parity` to complete.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity) {
  if (bar_try(b, parity)) return true;
  const uint64_t t0 = now_ns();
  while (!bar_try(b, parity))
    if (now_ns() - t0 > kWaitNs) return false;
  return true;
}
// Bulk copy of `bytes` (multiple of 16, 16-byte aligned ends) into this CTA's
// shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// bulk_load of bytes [off, off + bytes) of the two-segment string lo[0..split) ++ hi[0..).
__device__ __forceinline__ void bulk_load_split(void* dst, const char* lo, const char* hi, int64_t split,
                                                int64_t off, uint32_t bytes, uint64_t* bar) {
  if (off + bytes <= split) {
    bulk_load(dst, lo + off, bytes, bar);
  } else if (off >= split) {
    bulk_load(dst, hi + (off - split), bytes, bar);
  } else {  // the boundary falls inside this copy
    const uint32_t b0 = (uint32_t)(split - off);
    bulk_load(dst, lo + off, b0, bar);
    bulk_load(static_cast<char*>(dst) + b0, hi, bytes - b0, bar);
  }
}

// Bulk copy of `bytes` (multiple of 16, 16-byte aligned ends) from this CTA's
// shared memory to global memory, as one member of the current bulk group.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store has read its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Consumer side: every lane of the warp has finished reading the stage; one
// arrival per warp (the empty barrier counts warps).
__device__ __forceinline__ void warp_release(uint64_t* b) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) bar_arrive(b);
}

// Iteration state of one side of a ring of `nst` stages.
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int nst) {
    if (++stage == nst) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

// Producer warp: lane 0 waits (bounded) until the consumers have released
// stage r.stage (nothing to wait for while the ring is first being filled);
// the outcome is broadcast to the warp. `lane` = lane index in the warp.
__device__ __forceinline__ bool warp_acquire(uint64_t* empty, Ring r, int64_t filled, int nst, int lane) {
  if (filled < nst) return true;
  bool ok = true;
  if (lane == 0) ok = bar_wait(empty + r.stage, r.phase ^ 1u);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Producer side: after a failed acquire, wait for the last stages it filled
// (their copies) before returning. `filled` = number of stages filled so far.
__device__ __forceinline__ void producer_drain(uint64_t* full, int nst, Ring r, int64_t filled) {
  for (int i = 0; i < nst && i < filled; ++i) {
    // step back one stage
    if (r.stage == 0) {
      r.stage = nst - 1;
      r.phase ^= 1u;
    } else {
      --r.stage;
    }
    (void)bar_wait(full + r.stage, r.phase);
  }
}

}  // namespace pipe
}  // namespace gsec
