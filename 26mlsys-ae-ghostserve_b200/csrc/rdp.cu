// rdp.cu — Row-Diagonal Parity (Corbett et al., "Row-Diagonal Parity for Double
// Disk Failure Correction", FAST 2004) over KV shards.
//
// Geometry (p prime, k <= p-1 data shards): every shard is cut into stripes of
// (p-1) units of `unit` bytes.  In a stripe, cell (r, c) is unit r of column c,
// r in [0, p-2]; columns 0..p-2 are data (columns k..p-2 are virtual all-zero
// shards, i.e. the shortened code), column p-1 is the row parity P and column p
// the diagonal parity Q.
//   P[r]  = XOR_{c=0}^{p-2} D[r][c]
//   cell (r, c) for c in [0, p-1] lies on diagonal (r + c) mod p;
//   Q[d]  = XOR of the cells of diagonal d, d in [0, p-2] (diagonal p-1 is not stored).
// Diagonal arithmetic is per unit, so a thread owning byte lane b of a stripe
// XORs whole 16-byte vectors of cells; with p a template parameter every
// (r + c) mod p is a compile-time register index.
//
// Decode of up to two erased columns: one pass over the surviving cells of a
// stripe accumulates row syndromes R[r] (XOR over surviving columns 0..p-1) and
// diagonal syndromes S[d] (same over diagonal d, plus Q[d] if Q survives).
// Each erased cell is a fixed XOR of syndromes that depends only on which
// columns are erased; the host solves that GF(2) system once per call and passes
// one bit mask per erased cell.
#include <vector>

#include "common.cuh"
#include "pipe.cuh"
#include "rdp.cuh"

namespace gsec {
namespace {

__device__ __forceinline__ const char* seg(const char* lo, const char* hi, int64_t split, int64_t x) {
  return x < split ? lo + x : hi + (x - split);
}
__device__ __forceinline__ char* seg(char* lo, char* hi, int64_t split, int64_t x) {
  return x < split ? lo + x : hi + (x - split);
}
__device__ __forceinline__ uint4 ld16(const char* p) {
  uint4 v;
  asm("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ void st16(char* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------- encode ----
template <int P>
__global__ void __launch_bounds__(256) rdp_encode_kernel(const RdpEncodeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t lanes = a.unit >> 4;
  const int64_t stripe_bytes = (int64_t)(P - 1) * a.unit;
  const int64_t items = (a.s_end - a.s_begin) * lanes;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < items; g += step) {
    const int64_t stripe = a.s_begin + g / lanes;
    const int64_t lane = g - (stripe - a.s_begin) * lanes;
    const int64_t base = stripe * stripe_bytes + (lane << 4);
    const bool full = (stripe + 1) * stripe_bytes <= a.data_bytes;
    uint4 q[P];
#pragma unroll
    for (int d = 0; d < P; ++d) q[d] = vzero();
#pragma unroll
    for (int r = 0; r < P - 1; ++r) {
      const int64_t off = base + (int64_t)r * a.unit;
      uint4 x[P - 1];
#pragma unroll
      for (int c = 0; c < P - 1; ++c) {
        x[c] = vzero();
        if (c < a.k && (full || off < a.data_bytes)) x[c] = ld16(seg(a.d_lo[c], a.d_hi[c], a.split, off));
      }
      uint4 prow = vzero();
#pragma unroll
      for (int c = 0; c < P - 1; ++c) {
        prow = vxor(prow, x[c]);
        if ((r + c) % P != P - 1) q[(r + c) % P] = vxor(q[(r + c) % P], x[c]);
      }
      st16(a.parity[0] + off, prow);
      if ((r + P - 1) % P != P - 1) q[(r + P - 1) % P] = vxor(q[(r + P - 1) % P], prow);
    }
#pragma unroll
    for (int d = 0; d < P - 1; ++d) st16(a.parity[1] + base + (int64_t)d * a.unit, q[d]);
  }
}

// ------------------------------------------------------- encode (TMA ring) --
// Same arithmetic as rdp_encode_kernel, with the data cells staged in shared
// memory by bulk copies.  Work item = (stripe, 1 KiB segment of the unit);
// one ring stage = row r of the item's k data cells (k x 1 KiB).  64 consumer
// threads own 16-byte lanes of the segment; a 32-thread producer warp (one
// active lane) keeps kStages rows in flight.
constexpr int kSeg = 1024;
constexpr int kSegLanes = kSeg / 16;
static __device__ unsigned g_rdp_status;

template <int P>
__global__ void __launch_bounds__(kSegLanes + 32) rdp_encode_tma_kernel(const RdpEncodeArgs a, int nst) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int k = a.k;
  const int stage_bytes = k * kSeg;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nst * stage_bytes);
  uint64_t* empty = full + nst;
  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      pipe::bar_init(full + s, 1);
      pipe::bar_init(empty + s, kSegLanes / 32);
    }
    pipe::bar_init_fence();
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
  const int64_t spu = a.unit / kSeg;
  const int64_t items = (a.s_end - a.s_begin) * spu;
  const int64_t sb = (int64_t)(P - 1) * a.unit;

  if (threadIdx.x >= kSegLanes) {  // producer warp: lane c copies column c of each stage
    const int pl = threadIdx.x - kSegLanes;
    const bool mine = pl < k;
    const char* my_lo = mine ? a.d_lo[pl] : nullptr;
    const char* my_hi = mine ? a.d_hi[pl] : nullptr;
    pipe::Ring r;
    int64_t filled = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
      const int64_t stripe = a.s_begin + it / spu;
      const int64_t seg0 = (it % spu) * kSeg;
      for (int row = 0; row < P - 1; ++row) {
        if (!pipe::warp_acquire(empty, r, filled, nst, pl)) {
          if (pl == 0) {
            atomicOr(&g_rdp_status, 1u);
            pipe::producer_drain(full, nst, r, filled);
          }
          return;
        }
        const int64_t off = stripe * sb + (int64_t)row * a.unit + seg0;
        int64_t bytes = a.data_bytes - off;
        bytes = bytes < 0 ? 0 : (bytes > kSeg ? kSeg : bytes);
        if (pl == 0) pipe::bar_expect_tx(full + r.stage, (uint32_t)(bytes * k));
        __syncwarp();
        if (mine && bytes > 0)
          pipe::bulk_load_split(smem + (size_t)r.stage * stage_bytes + pl * kSeg, my_lo, my_hi, a.split, off,
                                (uint32_t)bytes, full + r.stage);
        r.next(nst);
        ++filled;
      }
    }
    return;
  }

  const int lane = threadIdx.x;
  pipe::Ring r;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t stripe = a.s_begin + it / spu;
    const int64_t base = stripe * sb + (it % spu) * kSeg + lane * 16;
    uint4 q[P];
#pragma unroll
    for (int d = 0; d < P; ++d) q[d] = vzero();
#pragma unroll
    for (int row = 0; row < P - 1; ++row) {
      if (!pipe::bar_wait(full + r.stage, r.phase)) {
        atomicOr(&g_rdp_status, 2u);
        return;
      }
      const int64_t off = base + (int64_t)row * a.unit;
      const uint4* st = reinterpret_cast<const uint4*>(smem + (size_t)r.stage * stage_bytes) + lane;
      const bool in_data = off < a.data_bytes;
      uint4 prow = vzero();
#pragma unroll
      for (int c = 0; c < P - 1; ++c) {
        if (c < k && in_data) {
          const uint4 x = st[c * kSegLanes];
          prow = vxor(prow, x);
          if ((row + c) % P != P - 1) q[(row + c) % P] = vxor(q[(row + c) % P], x);
        }
      }
      pipe::warp_release(empty + r.stage);
      r.next(nst);
      st16(a.parity[0] + off, prow);
      if ((row + P - 1) % P != P - 1) q[(row + P - 1) % P] = vxor(q[(row + P - 1) % P], prow);
    }
#pragma unroll
    for (int d = 0; d < P - 1; ++d) st16(a.parity[1] + base + (int64_t)d * a.unit, q[d]);
  }
}

// ---------------------------------------------------------------- decode ----
template <int P>
__global__ void __launch_bounds__(256) rdp_decode_kernel(const RdpDecodeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int NS = 2 * (P - 1);
  const int64_t lanes = a.unit >> 4;
  const int64_t stripe_bytes = (int64_t)(P - 1) * a.unit;
  const int64_t items = (a.s_end - a.s_begin) * lanes;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < items; g += step) {
    const int64_t stripe = a.s_begin + g / lanes;
    const int64_t lane = g - (stripe - a.s_begin) * lanes;
    const int64_t base = stripe * stripe_bytes + (lane << 4);
    const bool full = (stripe + 1) * stripe_bytes <= a.data_bytes;
    uint4 syn[NS];  // [0, P-1): row syndromes R[r]; [P-1, NS): diagonal syndromes S[d]
#pragma unroll
    for (int j = 0; j < NS; ++j) syn[j] = vzero();
#pragma unroll
    for (int c = 0; c <= P; ++c) {
      if (!((a.alive >> c) & 1u)) continue;
      const bool is_data = c < P - 1;
#pragma unroll
      for (int r = 0; r < P - 1; ++r) {
        const int64_t off = base + (int64_t)r * a.unit;
        if (is_data && !(full || off < a.data_bytes)) continue;
        const uint4 v = ld16(seg(a.lo[c], a.hi[c], a.split, off));
        if (c <= P - 1) {
          syn[r] = vxor(syn[r], v);
          if ((r + c) % P != P - 1) syn[(P - 1) + (r + c) % P] = vxor(syn[(P - 1) + (r + c) % P], v);
        } else {
          syn[(P - 1) + r] = vxor(syn[(P - 1) + r], v);
        }
      }
    }
    for (int e = 0; e < a.nout; ++e) {
      const bool out_data = a.out_col[e] < P - 1;
#pragma unroll
      for (int r = 0; r < P - 1; ++r) {
        const int64_t off = base + (int64_t)r * a.unit;
        const uint32_t m = a.mask[e][r];
        uint4 o = vzero();
#pragma unroll
        for (int j = 0; j < NS; ++j)
          if ((m >> j) & 1u) o = vxor(o, syn[j]);
        if (!out_data || off < a.data_bytes) st16(seg(a.out_lo[e], a.out_hi[e], a.split, off), o);
      }
    }
  }
}

// ------------------------------------------------------- decode (TMA ring) --
// rdp_decode_kernel's syndrome decode with the surviving cells staged in shared
// memory: one ring stage = row r of every surviving column of the item
// (stripe, 1 KiB segment), packed in column order.
// Warps of one CTA: 0-1 accumulate syndromes (one 16-byte lane column of the
// 1 KiB segment each), 2-3 write the erased cells, 4 issues the bulk copies.
constexpr int kDecThreads = 2 * kSegLanes + 32;

template <int P>
__global__ void __launch_bounds__(kDecThreads) rdp_decode_tma_kernel(const RdpDecodeArgs a, int nst) {
  constexpr int NS = 2 * (P - 1);
  extern __shared__ __align__(128) unsigned char smem[];
  const int nalive = __popc(a.alive);
  const int stage_bytes = nalive * kSeg;
  // After the ring: two syndrome buffers [2][NS][kSegLanes] handed from the
  // accumulating warps to the writing warps, so an item's erased cells are
  // written while the next item's rows are being accumulated.
  uint4* synsm = reinterpret_cast<uint4*>(smem + (size_t)nst * stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nst * stage_bytes + (size_t)2 * NS * kSeg);
  uint64_t* empty = full + nst;
  uint64_t* sfull = empty + nst;  // [2]: syndromes of an item are in the buffer
  uint64_t* sempty = sfull + 2;   // [2]: the writers are done with the buffer
  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      pipe::bar_init(full + s, 1);
      pipe::bar_init(empty + s, kSegLanes / 32);
    }
    for (int b = 0; b < 2; ++b) {
      pipe::bar_init(sfull + b, kSegLanes / 32);
      pipe::bar_init(sempty + b, kSegLanes / 32);
    }
    pipe::bar_init_fence();
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
  const int64_t spu = a.unit / kSeg;
  const int64_t items = (a.s_end - a.s_begin) * spu;
  const int64_t sb = (int64_t)(P - 1) * a.unit;

  if (threadIdx.x >= 2 * kSegLanes) {  // producer warp: lane j copies the j-th alive column
    const int pl = threadIdx.x - 2 * kSegLanes;
    int col = -1;
    for (uint32_t live = a.alive, j = 0; live; live &= live - 1u, ++j)
      if ((int)j == pl) col = __ffs(live) - 1;
    const char* my_lo = col >= 0 ? a.lo[col] : nullptr;
    const char* my_hi = col >= 0 ? a.hi[col] : nullptr;
    const bool my_data = col >= 0 && col < P - 1;
    const uint32_t ndata = __popc(a.alive & ((1u << (P - 1)) - 1u));  // alive data columns
    const uint32_t npar = (uint32_t)nalive - ndata;                   // alive P / Q
    pipe::Ring r;
    int64_t filled = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
      const int64_t stripe = a.s_begin + it / spu;
      const int64_t seg0 = (it % spu) * kSeg;
      for (int row = 0; row < P - 1; ++row) {
        if (!pipe::warp_acquire(empty, r, filled, nst, pl)) {
          if (pl == 0) {
            atomicOr(&g_rdp_status, 4u);
            pipe::producer_drain(full, nst, r, filled);
          }
          return;
        }
        const int64_t off = stripe * sb + (int64_t)row * a.unit + seg0;
        int64_t dbytes = a.data_bytes - off;
        dbytes = dbytes < 0 ? 0 : (dbytes > kSeg ? kSeg : dbytes);
        if (pl == 0) pipe::bar_expect_tx(full + r.stage, ndata * (uint32_t)dbytes + npar * (uint32_t)kSeg);
        __syncwarp();
        const int64_t bytes = my_data ? dbytes : kSeg;
        if (col >= 0 && bytes > 0)
          pipe::bulk_load_split(smem + (size_t)r.stage * stage_bytes + pl * kSeg, my_lo, my_hi, a.split, off,
                                (uint32_t)bytes, full + r.stage);
        r.next(nst);
        ++filled;
      }
    }
    return;
  }

  if (threadIdx.x >= kSegLanes) {  // writer warps: the erased cells as a chain program
    const int lane = threadIdx.x - kSegLanes;
    pipe::Ring sb_r;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
      if (!pipe::bar_wait(sfull + sb_r.stage, sb_r.phase)) {
        atomicOr(&g_rdp_status, 16u);
        return;
      }
      const uint4* syn = synsm + (size_t)sb_r.stage * NS * kSegLanes + lane;
      const int64_t stripe = a.s_begin + it / spu;
      const int64_t base = stripe * sb + (it % spu) * kSeg + lane * 16;
      uint4 o = vzero();
      for (int t = 0; t < a.nprog; ++t) {
        if (!a.prog_chain[t]) o = vzero();
        for (uint32_t dm = a.prog_diff[t]; dm; dm &= dm - 1u) o = vxor(o, syn[(__ffs(dm) - 1) * kSegLanes]);
        const int e = a.prog_out[t] >> 4;
        const int64_t off = base + (int64_t)(a.prog_out[t] & 15) * a.unit;
        if (a.out_col[e] >= P - 1 || off < a.data_bytes) st16(seg(a.out_lo[e], a.out_hi[e], a.split, off), o);
      }
      pipe::warp_release(sempty + sb_r.stage);
      sb_r.next(2);
    }
    return;
  }

  const int lane = threadIdx.x;
  int pos[P + 1];  // slot of column c inside a stage
#pragma unroll
  for (int c = 0; c <= P; ++c) pos[c] = __popc(a.alive & ((1u << c) - 1u)) * kSegLanes;
  pipe::Ring r;
  pipe::Ring sb_r;
  int64_t handed = 0;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t stripe = a.s_begin + it / spu;
    const int64_t base = stripe * sb + (it % spu) * kSeg + lane * 16;
    uint4 syn[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) syn[j] = vzero();
#pragma unroll
    for (int row = 0; row < P - 1; ++row) {
      if (!pipe::bar_wait(full + r.stage, r.phase)) {
        atomicOr(&g_rdp_status, 8u);
        return;
      }
      const int64_t off = base + (int64_t)row * a.unit;
      const bool in_data = off < a.data_bytes;
      const uint4* st = reinterpret_cast<const uint4*>(smem + (size_t)r.stage * stage_bytes) + lane;
#pragma unroll
      for (int c = 0; c <= P; ++c) {
        if (!((a.alive >> c) & 1u)) continue;
        if (c < P - 1 && !in_data) continue;
        const uint4 v = st[pos[c]];
        if (c <= P - 1) {
          syn[row] = vxor(syn[row], v);
          if ((row + c) % P != P - 1) syn[(P - 1) + (row + c) % P] = vxor(syn[(P - 1) + (row + c) % P], v);
        } else {
          syn[(P - 1) + row] = vxor(syn[(P - 1) + row], v);
        }
      }
      pipe::warp_release(empty + r.stage);
      r.next(nst);
    }
    // hand the syndromes to the writers (wait until they are done with the buffer)
    if (handed >= 2 && !pipe::bar_wait(sempty + sb_r.stage, sb_r.phase ^ 1u)) {
      atomicOr(&g_rdp_status, 32u);
      return;
    }
    uint4* dst = synsm + (size_t)sb_r.stage * NS * kSegLanes + lane;
#pragma unroll
    for (int j = 0; j < NS; ++j) dst[j * kSegLanes] = syn[j];
    pipe::warp_release(sfull + sb_r.stage);
    sb_r.next(2);
    ++handed;
  }
}

template <typename K>
int grid_for(K kernel, int threads, int64_t items) {
  LaunchCache& cache = launch_cache();
  int per_sm = cache.blocks_per_sm(kernel, threads, 0);
  if (per_sm < 1) per_sm = 1;
  int64_t grid = (int64_t)sm_count() * per_sm;
  const int64_t need = (items + threads - 1) / threads;
  if (need < grid) grid = need;
  return (int)(grid < 1 ? 1 : grid);
}

#ifndef GSEC_RDP_STAGES
#define GSEC_RDP_STAGES 3
#endif
#ifndef GSEC_RDP_CTAS
#define GSEC_RDP_CTAS 5
#endif
#ifndef GSEC_RDP_DEC_STAGES
#define GSEC_RDP_DEC_STAGES 4
#endif
constexpr int kStages = GSEC_RDP_STAGES;   // ring stages per CTA
constexpr int kDecStages = GSEC_RDP_DEC_STAGES;  // the decode's (its items end in a burst of stores)
constexpr int kCtasPerSm = GSEC_RDP_CTAS;  // resident CTAs per SM (at most)

// p = 3 (two rows per stripe): the register kernels, each thread streaming one
// 16-byte lane of a stripe with all its cells' loads in flight, beat the
// staging ring, whose per-item hand-offs dominate such short items (decode of
// 16 MiB shards: 0.60 -> 1.07 of the copy peak, 64 MiB: 0.70 -> 0.91; encode
// of 2 MiB shards 0.50 -> 0.61). From p = 5 on the ring is faster, and so it
// is for inputs in another GPU's memory (bulk copies over NVLink outrun
// 16-byte loads there).
#ifndef GSEC_RDP_REG_DECODE_MAXP
#define GSEC_RDP_REG_DECODE_MAXP 3
#endif
#ifndef GSEC_RDP_REG_ENCODE_MAXP
#define GSEC_RDP_REG_ENCODE_MAXP 3
#endif
template <int P>
int launch_encode(const RdpEncodeArgs& a, cudaStream_t s) {
  if (a.unit % kSeg == 0 && (P > GSEC_RDP_REG_ENCODE_MAXP || a.remote)) {  // TMA ring: units split into whole 1 KiB segments
    LaunchCache& cache = launch_cache();
    auto k = rdp_encode_tma_kernel<P>;
    // small k makes small stages: keep ~18 KiB of loads in flight per CTA all the same
    int nst = 18 / a.k;
    nst = nst < kStages ? kStages : (nst > 9 ? 9 : nst);
    const size_t smem = (size_t)nst * a.k * kSeg + 2 * (size_t)nst * sizeof(uint64_t);
    int per_sm = cache.blocks_per_sm(k, kSegLanes + 32, smem);
    if (per_sm < 0) return check_launch("rdp_encode_tma launch shape");
    per_sm = per_sm > kCtasPerSm ? kCtasPerSm : per_sm;
    const int64_t items = (a.s_end - a.s_begin) * (a.unit / kSeg);
    const int64_t grid = balanced_grid(items, (int64_t)sm_count() * per_sm);
    return launch_rc(launch_pdl(k, dim3((unsigned)grid), dim3(kSegLanes + 32), smem, s, a, nst),
                     "rdp_encode_tma_kernel");
  }
  const int64_t items = (a.s_end - a.s_begin) * (a.unit >> 4);
  const int threads = 256;
  const int grid = grid_for(rdp_encode_kernel<P>, threads, items);
  if (const cudaError_t lrc = launch_pdl(rdp_encode_kernel<P>, dim3((unsigned)(grid)), dim3(threads), 0, s, a))
    return launch_rc(lrc, "rdp_encode_kernel");
  return check_launch("rdp_encode_kernel");
}
template <int P>
int launch_decode(const RdpDecodeArgs& a, cudaStream_t s) {
  if (a.unit % kSeg == 0 && (P > GSEC_RDP_REG_DECODE_MAXP || a.remote)) {
    LaunchCache& cache = launch_cache();
    auto k = rdp_decode_tma_kernel<P>;
    const int nalive = __builtin_popcount(a.alive);
    int nst = 24 / nalive;  // ~24 KiB of loads in flight per CTA
    nst = nst < kDecStages ? kDecStages : (nst > 12 ? 12 : nst);
    const size_t smem = (size_t)nst * nalive * kSeg + (size_t)2 * 2 * (P - 1) * kSeg +
                        (2 * (size_t)nst + 4) * sizeof(uint64_t);
    int per_sm = cache.blocks_per_sm(k, kDecThreads, smem);
    if (per_sm < 0) return check_launch("rdp_decode_tma launch shape");
    // p = 3: two rows per item, so an item's fixed hand-off latency dominates;
    // more resident CTAs keep more items in flight (measured: 0.51 -> 0.60 of
    // the copy peak at 16 MiB shards, 0.58 -> 0.70 at 64 MiB; larger p gain nothing)
    const int cap = P <= 3 ? 2 * kCtasPerSm : kCtasPerSm;
    per_sm = per_sm > cap ? cap : per_sm;
    const int64_t items = (a.s_end - a.s_begin) * (a.unit / kSeg);
    const int64_t grid = balanced_grid(items, (int64_t)sm_count() * per_sm);
    return launch_rc(launch_pdl(k, dim3((unsigned)grid), dim3(kDecThreads), smem, s, a, nst),
                     "rdp_decode_tma_kernel");
  }
  const int64_t items = (a.s_end - a.s_begin) * (a.unit >> 4);
  const int threads = 256;
  const int grid = grid_for(rdp_decode_kernel<P>, threads, items);
  if (const cudaError_t lrc = launch_pdl(rdp_decode_kernel<P>, dim3((unsigned)(grid)), dim3(threads), 0, s, a))
    return launch_rc(lrc, "rdp_decode_kernel");
  return check_launch("rdp_decode_kernel");
}

}  // namespace

unsigned rdp_device_status(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_rdp_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_rdp_status, &z, sizeof(z));
  }
  return v;
}

bool rdp_prime_supported(int p) {
  return p == 3 || p == 5 || p == 7 || p == 11 || p == 13 || p == 17;
}

int rdp_encode(const RdpEncodeArgs& a, cudaStream_t s) {
  if (a.s_end <= a.s_begin) return GSEC_OK;
  switch (a.p) {
    case 3: return launch_encode<3>(a, s);
    case 5: return launch_encode<5>(a, s);
    case 7: return launch_encode<7>(a, s);
    case 11: return launch_encode<11>(a, s);
    case 13: return launch_encode<13>(a, s);
    case 17: return launch_encode<17>(a, s);
    default: set_error("RDP prime p=%d not supported (3,5,7,11,13,17)", a.p); return GSEC_EUNSUPPORTED;
  }
}

int rdp_decode(const RdpDecodeArgs& a, cudaStream_t s) {
  if (a.s_end <= a.s_begin || a.nout == 0) return GSEC_OK;
  switch (a.p) {
    case 3: return launch_decode<3>(a, s);
    case 5: return launch_decode<5>(a, s);
    case 7: return launch_decode<7>(a, s);
    case 11: return launch_decode<11>(a, s);
    case 13: return launch_decode<13>(a, s);
    case 17: return launch_decode<17>(a, s);
    default: set_error("RDP prime p=%d not supported (3,5,7,11,13,17)", a.p); return GSEC_EUNSUPPORTED;
  }
}

// Solve the erased cells of one stripe as XORs of syndromes.
//   cols: erased columns in [0, p] (p-1 = row parity, p = diagonal parity).
// Unknown u = e*(p-1) + r is cell (r, cols[e]).  Syndrome ids: r for R[r],
// (p-1)+d for S[d].  Equations (over GF(2)):
//   row r      : XOR_{e: cols[e] <= p-1} x(e, r)                           = R[r]
//   diagonal d : XOR_{e: cols[e] <= p-1, r=(d-cols[e]) mod p, r<p-1} x(e, r)
//                ^ [Q erased] x(Q, d)                                       = S[d]
int rdp_solve_masks(int p, const int* cols, int ncols, uint32_t mask[2][16]) {
  const int rows = p - 1;
  const int nunk = ncols * rows;
  const int neq = 2 * rows;
  std::vector<uint64_t> lhs(neq, 0);
  std::vector<uint32_t> rhs(neq, 0);
  for (int r = 0; r < rows; ++r) {
    rhs[r] = 1u << r;
    for (int e = 0; e < ncols; ++e)
      if (cols[e] <= p - 1) lhs[r] |= 1ull << (e * rows + r);
  }
  for (int d = 0; d < rows; ++d) {
    const int q = rows + d;
    rhs[q] = 1u << q;
    for (int e = 0; e < ncols; ++e) {
      if (cols[e] <= p - 1) {
        const int r = ((d - cols[e]) % p + p) % p;
        if (r < rows) lhs[q] |= 1ull << (e * rows + r);
      } else {
        lhs[q] |= 1ull << (e * rows + d);
      }
    }
  }
  // Gauss-Jordan over GF(2): pivot on each unknown in turn.
  std::vector<int> pivot_of(nunk, -1);
  std::vector<bool> used(neq, false);
  for (int u = 0; u < nunk; ++u) {
    int piv = -1;
    for (int i = 0; i < neq; ++i)
      if (!used[i] && ((lhs[i] >> u) & 1ull)) { piv = i; break; }
    if (piv < 0) {
      set_error("RDP erasure pattern is not decodable (singular system)");
      return GSEC_EUNRECOVERABLE;
    }
    used[piv] = true;
    pivot_of[u] = piv;
    for (int i = 0; i < neq; ++i)
      if (i != piv && ((lhs[i] >> u) & 1ull)) { lhs[i] ^= lhs[piv]; rhs[i] ^= rhs[piv]; }
  }
  for (int e = 0; e < ncols; ++e)
    for (int r = 0; r < rows; ++r) mask[e][r] = rhs[pivot_of[e * rows + r]];
  return GSEC_OK;
}

// Greedy chain over the erased cells: each step takes the unsolved cell whose
// syndrome set differs least from the previous step's (reusing that cell), or
// starts afresh when that is cheaper. For two erased data columns this finds
// RDP's alternating row/diagonal recovery chains: one syndrome per cell after
// the first.
void rdp_build_program(RdpDecodeArgs& a) {
  const int rows = a.p - 1;
  const int n = a.nout * rows;
  bool done[32] = {};
  uint32_t prev = 0;
  bool have_prev = false;
  for (int t = 0; t < n; ++t) {
    int best = -1, best_cost = 1 << 30;
    bool best_chain = false;
    for (int u = 0; u < n; ++u) {
      if (done[u]) continue;
      const uint32_t m = a.mask[u / rows][u % rows];
      const int fresh = __builtin_popcount(m);
      const int chained = have_prev ? __builtin_popcount(m ^ prev) : 1 << 30;
      const int cost = chained <= fresh ? chained : fresh;
      if (cost < best_cost) {
        best = u;
        best_cost = cost;
        best_chain = chained <= fresh;
      }
    }
    const uint32_t m = a.mask[best / rows][best % rows];
    done[best] = true;
    a.prog_out[t] = (uint8_t)(((best / rows) << 4) | (best % rows));
    a.prog_chain[t] = best_chain ? 1 : 0;
    a.prog_diff[t] = best_chain ? (m ^ prev) : m;
    prev = m;
    have_prev = true;
  }
  a.nprog = n;
}

}  // namespace gsec
