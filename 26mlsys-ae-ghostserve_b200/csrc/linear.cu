// linear.cu — kernels for position-wise linear codes (XOR, GF(2^8), GF(2^16)).
//
// Layout assumed by the vector kernels: every shard pointer 16-byte aligned and
// `split`/`begin` multiples of 16, so each thread moves whole 16-byte vectors
// that never straddle a segment boundary.  Anything else goes to the scalar
// kernel (same arithmetic, one symbol per thread).
//
// GF constant multiplication uses a 256-entry table per input shard in shared
// memory.  Entry x of input i packs the products coef[j][i]*x of all outputs j
// (one byte each for GF(2^8), one u16 for GF(2^16) split into low/high byte
// tables), so one shared-memory load serves every parity shard.  Each table is
// replicated R times and lane l reads copy l % R: with R = 32 the 32 lanes of a
// warp always hit 32 different banks whatever the data bytes are.
//
// The RS(k, m <= 2) encode itself (coefficients = the Cauchy generator) skips
// the tables: gf8_cauchy_kernel transposes 32-byte groups into bit planes and
// runs the generator as a compile-time XOR network (cauchy_net.cuh), about 60 %
// of the table kernel's instructions per byte.
#include "linear.cuh"
#include "cauchy_net.cuh"
#include "pipe.cuh"

namespace gsec {
namespace {

__device__ __forceinline__ const char* seg(const char* lo, const char* hi, int64_t split,
                                           int64_t x) {
  return x < split ? lo + x : hi + (x - split);
}
__device__ __forceinline__ char* seg(char* lo, char* hi, int64_t split, int64_t x) {
  return x < split ? lo + x : hi + (x - split);
}

// Plain (coherent) 16-byte load with no L1 allocation: shards are streamed once,
// and the pointer may be a peer GPU's memory mapped over NVLink.
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

// Sub-vector tail [t0, end) of every output, one thread, symbol at a time.
__device__ void linear_tail(const LinearPass& a, int64_t t0) {
  if (a.field == Field::GF16) {
    for (int64_t x = t0; x + 2 <= a.end; x += 2) {
      for (int j = 0; j < a.nout; ++j) {
        uint32_t acc = 0;
        for (int i = 0; i < a.nin; ++i) {
          const uint16_t w = *reinterpret_cast<const uint16_t*>(seg(a.in_lo[i], a.in_hi[i], a.split, x));
          acc ^= gf16_mul(w, a.coef[j][i]);
        }
        if (x < a.out_end[j])
          *reinterpret_cast<uint16_t*>(seg(a.out_lo[j], a.out_hi[j], a.split, x)) = (uint16_t)acc;
      }
    }
    return;
  }
  for (int64_t x = t0; x < a.end; ++x) {
    for (int j = 0; j < a.nout; ++j) {
      uint32_t acc = 0;
      for (int i = 0; i < a.nin; ++i) {
        const uint8_t b = *reinterpret_cast<const uint8_t*>(seg(a.in_lo[i], a.in_hi[i], a.split, x));
        acc ^= (a.field == Field::XOR) ? b : gf8_mul(b, a.coef[j][i] & 0xffu);
      }
      if (x < a.out_end[j]) *reinterpret_cast<uint8_t*>(seg(a.out_lo[j], a.out_hi[j], a.split, x)) = (uint8_t)acc;
    }
  }
}

// ------------------------------------------------------- XOR (TMA ring) -----
// Work item = one 1 KiB segment of the range; a ring stage holds that segment
// of every input (nin x 1 KiB), filled by bulk copies from a producer lane and
// XORed by 64 consumer threads (16 bytes each), which store every output.
constexpr int kLSeg = 1024;
constexpr int kLLanes = kLSeg / 16;
constexpr int kLStages = 3;          // at least; narrow passes get more (see ring_stages)
constexpr int kLRingBytes = 18 * 1024;  // bytes in flight per CTA the ring aims for
static __device__ unsigned g_linear_status;

// SPS 1 KiB segments of every input per stage: passes with few inputs take
// several segments at once so the fixed cost of a stage (barrier wait and
// release) is spread over more bytes.
template <int SPS>
__global__ void __launch_bounds__(kLLanes + 32) xor_tma_kernel(const LinearPass a, int nst) {
  constexpr int ITEM = SPS * kLSeg;  // bytes of each input per stage
  extern __shared__ __align__(128) unsigned char smem[];
  const int nin = a.nin;
  const int stage_bytes = nin * ITEM;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nst * stage_bytes);
  uint64_t* empty = full + nst;
  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      pipe::bar_init(full + s, 1);
      pipe::bar_init(empty + s, kLLanes / 32);
    }
    pipe::bar_init_fence();
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
  const int64_t vend = a.begin + (((a.end - a.begin) >> 4) << 4);  // end of the whole-vector part
  const int64_t items = (vend - a.begin + ITEM - 1) / ITEM;

  if (threadIdx.x >= kLLanes) {  // producer warp: lane i copies input i of each stage
    const int pl = threadIdx.x - kLLanes;
    const bool mine = pl < nin;
    const char* my_lo = mine ? a.in_lo[pl] : nullptr;
    const char* my_hi = mine ? a.in_hi[pl] : nullptr;
    pipe::Ring r;
    int64_t filled = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
      if (!pipe::warp_acquire(empty, r, filled, nst, pl)) {
        if (pl == 0) {
          atomicOr(&g_linear_status, 1u);
          pipe::producer_drain(full, nst, r, filled);
        }
        return;
      }
      const int64_t off = a.begin + it * ITEM;
      const int64_t bytes = vend - off < ITEM ? vend - off : ITEM;
      if (pl == 0) pipe::bar_expect_tx(full + r.stage, (uint32_t)(bytes * nin));
      __syncwarp();
      if (mine)
        pipe::bulk_load_split(smem + (size_t)r.stage * stage_bytes + pl * ITEM, my_lo, my_hi, a.split, off,
                              (uint32_t)bytes, full + r.stage);
      r.next(nst);
      ++filled;
    }
    return;
  }

  const int lane = threadIdx.x;
  pipe::Ring r;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    if (!pipe::bar_wait(full + r.stage, r.phase)) {
      atomicOr(&g_linear_status, 2u);
      return;
    }
    const int64_t off0 = a.begin + it * ITEM + lane * 16;
    const uint4* st = reinterpret_cast<const uint4*>(smem + (size_t)r.stage * stage_bytes) + lane;
    uint4 acc[SPS];
#pragma unroll
    for (int q = 0; q < SPS; ++q) {
      acc[q] = vzero();
      if (off0 + q * kLSeg < vend)
        for (int i = 0; i < nin; ++i) acc[q] = vxor(acc[q], st[i * SPS * kLLanes + q * kLLanes]);
    }
    pipe::warp_release(empty + r.stage);
    r.next(nst);
#pragma unroll
    for (int q = 0; q < SPS; ++q) {
      const int64_t off = off0 + q * kLSeg;
      if (off < vend)
        for (int o = 0; o < a.nout; ++o)
          if (off + 16 <= a.out_end[o]) st16(seg(a.out_lo[o], a.out_hi[o], a.split, off), acc[q]);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, vend);
}

// Few XOR inputs (one: the parity is a copy, the mirror of a one-data-shard
// code): a plain streaming kernel with four independent 16-byte vectors of
// every input in flight per thread keeps more bytes in flight than a staging
// ring needs to; the ring kernel spends its time on barrier hand-offs here.
#ifndef GSEC_XOR_STREAM_MAXIN
#define GSEC_XOR_STREAM_MAXIN 3
#endif
template <int NIN>
__global__ void __launch_bounds__(256) xor_stream_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += 4 * step) {
    uint4 x[4][NIN];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int i = 0; i < NIN; ++i)
        if (v + u * step < nvec) x[u][i] = ld16(seg(a.in_lo[i], a.in_hi[i], a.split, a.begin + ((v + u * step) << 4)));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t off = a.begin + ((v + u * step) << 4);
      if (v + u * step < nvec) {
        uint4 acc = x[u][0];
#pragma unroll
        for (int i = 1; i < NIN; ++i) acc = vxor(acc, x[u][i]);
        for (int o = 0; o < a.nout; ++o)
          if (off + 16 <= a.out_end[o]) st16(seg(a.out_lo[o], a.out_hi[o], a.split, off), acc);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

template <int SPS>
int launch_xor(const LinearPass& a, cudaStream_t s, int ring_bytes) {
  // keep ring_bytes of loads in flight per CTA whatever the input count
  int nst = ring_bytes / (a.nin * SPS * kLSeg);
  nst = nst < kLStages ? kLStages : (nst > 18 ? 18 : nst);
  LaunchCache& cache = launch_cache();
  auto k = xor_tma_kernel<SPS>;
  const size_t smem = (size_t)nst * a.nin * SPS * kLSeg + 2 * (size_t)nst * sizeof(uint64_t);
  int per_sm = cache.blocks_per_sm(k, kLLanes + 32, smem);
  if (per_sm < 0) return check_launch("xor_tma launch shape");
  per_sm = per_sm > 5 ? 5 : per_sm;
  const int64_t items = ((a.end - a.begin) / 16 * 16 + SPS * kLSeg - 1) / (SPS * kLSeg);
  const int64_t grid = balanced_grid(items, (int64_t)sm_count() * per_sm);
  return launch_rc(launch_pdl(k, dim3((unsigned)grid), dim3(kLLanes + 32), smem, s, a, nst), "xor_tma_kernel");
}

// ------------------------------------------------- GF(2^8), fixed input count
// NIN a compile-time constant: every input's 16-byte vector is loaded before
// any lookup, table offsets are immediates, and the packed table words (byte j
// of an entry = output j's product) are XORed across inputs per data byte
// position; one 4x4 byte transpose per word then yields every output word.
// Tables: 256 u32 entries per input, replicated R times (lane l reads copy
// l % R); built once per CTA into a compact array, then fanned out with
// consecutive threads writing consecutive words (no bank conflicts).
// FLAT: single-segment shards and outputs that take the whole range (no
// per-vector segment select, no store bound check).
template <int NIN, bool FLAT>
__global__ void __launch_bounds__(1024) gf8_fixed_kernel(const LinearPass a) {
  constexpr int R = NIN <= 6 ? 32 : 16;
  constexpr int RSH = R == 32 ? 5 : 4;
  extern __shared__ __align__(128) uint32_t tab[];   // [NIN][256][R]
  uint32_t* compact = tab + NIN * 256 * R;           // [NIN][256]
  for (int e = threadIdx.x; e < NIN * 256; e += blockDim.x) {
    const int i = e >> 8, x = e & 255;
    uint32_t entry = 0;
    for (int j = 0; j < a.nout; ++j) entry |= gf8_mul((uint32_t)(a.coef[j][i] & 0xffu), (uint32_t)x) << (8 * j);
    compact[e] = entry;
  }
  __syncthreads();
  for (int w = threadIdx.x; w < NIN * 256 * R; w += blockDim.x) tab[w] = compact[w >> RSH];
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();

  // Byte offset of this lane's replica inside an entry; entries are R*4 bytes
  // apart, so (data byte << log2(R*4)) | lane_off addresses a lookup with one
  // shift and one LOP3, the table's base being an immediate per input.
  constexpr int ESH = RSH + 2;
  constexpr uint32_t EMASK = 0xffu << ESH;
  const uint32_t lane_off = (threadIdx.x & (R - 1)) * 4u;
  const unsigned char* tb = reinterpret_cast<const unsigned char*>(tab);
  const char* in_lo[NIN];
  const char* in_hi[NIN];
#pragma unroll
  for (int i = 0; i < NIN; ++i) {
    in_lo[i] = a.in_lo[i];
    in_hi[i] = a.in_hi[i];
  }
  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += step) {
    const int64_t off = a.begin + (v << 4);
    uint4 x[NIN];
#pragma unroll
    for (int i = 0; i < NIN; ++i) x[i] = ld16(FLAT ? in_lo[i] + off : seg(in_lo[i], in_hi[i], a.split, off));
    uint32_t acc[4][4];  // [word][byte position]
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[w][b] = 0u;
#pragma unroll
    for (int i = 0; i < NIN; ++i) {
      const unsigned char* t = tb + i * 256 * R * 4;
      const uint32_t xs[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t d = xs[w];
        acc[w][0] ^= *reinterpret_cast<const uint32_t*>(t + (((d << ESH) & EMASK) | lane_off));
        acc[w][1] ^= *reinterpret_cast<const uint32_t*>(t + (((d >> (8 - ESH)) & EMASK) | lane_off));
        acc[w][2] ^= *reinterpret_cast<const uint32_t*>(t + (((d >> (16 - ESH)) & EMASK) | lane_off));
        acc[w][3] ^= *reinterpret_cast<const uint32_t*>(t + (((d >> (24 - ESH)) & EMASK) | lane_off));
      }
    }
    uint32_t o[4][4];  // [output][word]
    const bool four = a.nout > 2;  // outputs 2 and 3 need the second half of the transpose
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t u = __byte_perm(acc[w][0], acc[w][1], 0x5140);
      const uint32_t q = __byte_perm(acc[w][2], acc[w][3], 0x5140);
      o[0][w] = __byte_perm(u, q, 0x5410);
      o[1][w] = __byte_perm(u, q, 0x7632);
      o[2][w] = o[3][w] = 0u;
      if (four) {
        const uint32_t u2 = __byte_perm(acc[w][0], acc[w][1], 0x7362);
        const uint32_t q2 = __byte_perm(acc[w][2], acc[w][3], 0x7362);
        o[2][w] = __byte_perm(u2, q2, 0x5410);
        o[3][w] = __byte_perm(u2, q2, 0x7632);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < a.nout && (FLAT || off + 16 <= a.out_end[j]))
        st16(FLAT ? a.out_lo[j] + off : seg(a.out_lo[j], a.out_hi[j], a.split, off),
             make_uint4(o[j][0], o[j][1], o[j][2], o[j][3]));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

// ------------------------------------ GF(2^8) encode, generator fixed at build
// Multiplying a byte by a constant c is a linear map over GF(2): bit r of c*x is
// the XOR of the bits s of x for which bit r of c*2^s is set. With the 32 bytes
// of a group transposed into 8 bit planes (word s = bit s of every byte), one
// output plane is a plain XOR of input planes, and with the code's generator
// known at compile time the choice of planes is a constant: the network
// (cauchy_net.cuh, written by gen_cauchy_net.py with the XOR pairs that several
// planes share computed once) is straight-line 3-input XORs, no tables, no
// lookups. Per 32-byte group of one input, its 8x8 bit transpose in every byte
// lane of 8 words (its own inverse) takes 60 integer instructions; the network
// takes about 0.65 per input byte for two parity rows. The generator is the Cauchy block C[j][i] = 1 / ((k + j) XOR i) over
// GF(2^8)/0x11d that the engine's RS(k, m) encode uses; passes with other
// coefficients (decode) keep the table kernel.
__host__ __device__ constexpr uint32_t cx_gf8_mul(uint32_t a, uint32_t b) {
  uint32_t acc = 0;
  while (b) {
    if (b & 1u) acc ^= a;
    a <<= 1;
    if (a & 0x100u) a ^= 0x11du;
    b >>= 1;
  }
  return acc;
}
__host__ __device__ constexpr uint32_t cx_gf8_inv(uint32_t a) {  // a^254 (a != 0)
  uint32_t r = 1, e = 254;
  while (e) {
    if (e & 1u) r = cx_gf8_mul(r, a);
    a = cx_gf8_mul(a, a);
    e >>= 1;
  }
  return r;
}
__host__ __device__ constexpr uint32_t cauchy_coef(int k, int j, int i) {
  return cx_gf8_inv((uint32_t)((k + j) ^ i));
}
// Exchange the bits of a under (m << s) with the bits of b under m.
__device__ __forceinline__ void swap_bits(uint32_t& a, uint32_t& b, int s, uint32_t m) {
  const uint32_t x = ((a >> s) ^ b) & m;
  b ^= x;
  a ^= x << s;
}
// Bit t of byte lane l of word s  <->  bit s of byte lane l of word t.
__device__ __forceinline__ void transpose8(uint32_t (&w)[8]) {
#pragma unroll
  for (int t = 0; t < 4; ++t) swap_bits(w[t], w[t + 4], 4, 0x0f0f0f0fu);
#pragma unroll
  for (int t = 0; t < 8; t += (t & 1) ? 3 : 1) swap_bits(w[t], w[t + 2], 2, 0x33333333u);
#pragma unroll
  for (int t = 0; t < 8; t += 2) swap_bits(w[t], w[t + 1], 1, 0x55555555u);
}

// FLAT: every shard is one segment and every output takes the whole range, so
// a lane's two vectors of a shard sit 512 bytes apart behind one pointer and
// no store needs a bound check (the bench's and the hook's encodes).
template <int K, int M, bool FLAT>
__global__ void __launch_bounds__(256, 3) gf8_cauchy_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  // A warp takes 1 KiB of every shard at a time; lane l transposes its vectors
  // l and l + 32 as one 32-byte group (any two vectors make a group), so every
  // load and store instruction covers 512 contiguous bytes.
  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t nchunk = (nvec + 63) >> 6;
  const int lane = threadIdx.x & 31;
  const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunk; c += nwarp) {
    const int64_t v0 = (c << 6) + lane;
    if (v0 >= nvec) continue;  // the last chunk's idle lanes
    const bool pair = v0 + 32 < nvec;
    const int64_t off0 = a.begin + (v0 << 4), off1 = off0 + 512;
    uint32_t w[K][8];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const char* p0 = FLAT ? a.in_lo[i] + off0 : seg(a.in_lo[i], a.in_hi[i], a.split, off0);
      const char* p1 = FLAT ? p0 + 512 : seg(a.in_lo[i], a.in_hi[i], a.split, off1);
      const uint4 x0 = ld16(p0);
      const uint4 x1 = pair ? ld16(p1) : vzero();
      w[i][0] = x0.x, w[i][1] = x0.y, w[i][2] = x0.z, w[i][3] = x0.w;
      w[i][4] = x1.x, w[i][5] = x1.y, w[i][6] = x1.z, w[i][7] = x1.w;
    }
#pragma unroll
    for (int i = 0; i < K; ++i) transpose8(w[i]);
    uint32_t o[M][8];
    CauchyNet<K, M>::run(w, o);
#pragma unroll
    for (int j = 0; j < M; ++j) {
      transpose8(o[j]);
      char* q0 = FLAT ? a.out_lo[j] + off0 : seg(a.out_lo[j], a.out_hi[j], a.split, off0);
      char* q1 = FLAT ? q0 + 512 : seg(a.out_lo[j], a.out_hi[j], a.split, off1);
      if (FLAT || off0 + 16 <= a.out_end[j]) st16(q0, make_uint4(o[j][0], o[j][1], o[j][2], o[j][3]));
      if (pair && (FLAT || off1 + 16 <= a.out_end[j])) st16(q1, make_uint4(o[j][4], o[j][5], o[j][6], o[j][7]));
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

// --------------------------------------------------------------- GF(2^8) ----
template <int NOUT, int R>
__global__ void __launch_bounds__(1024) gf8_vec_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ uint32_t tab[];  // [nin][256][R]
  for (int e = threadIdx.x; e < a.nin * 256; e += blockDim.x) {
    const int i = e >> 8, x = e & 255;
    uint32_t entry = 0;
#pragma unroll
    for (int j = 0; j < NOUT; ++j) entry |= gf8_mul((uint32_t)(a.coef[j][i] & 0xffu), (uint32_t)x) << (8 * j);
    uint32_t* dst = tab + (size_t)e * R;
#pragma unroll
    for (int r = 0; r < R; ++r) dst[r] = entry;
  }
  __syncthreads();
  const uint32_t* tl = tab + (threadIdx.x & (R - 1));

  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += step) {
    const int64_t off = a.begin + (v << 4);
    uint32_t o[NOUT][4];
#pragma unroll
    for (int j = 0; j < NOUT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0u;
#pragma unroll 2
    for (int i = 0; i < a.nin; ++i) {
      const uint4 xv = ld16(seg(a.in_lo[i], a.in_hi[i], a.split, off));
      const uint32_t* t = tl + (size_t)i * 256 * R;
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t x = xs[w];
        const uint32_t t0 = t[(x & 0xffu) * R];
        const uint32_t t1 = t[((x >> 8) & 0xffu) * R];
        const uint32_t t2 = t[((x >> 16) & 0xffu) * R];
        const uint32_t t3 = t[(x >> 24) * R];
        // 4x4 byte transpose: output j gets byte j of t0..t3 (the products of data bytes 0..3).
        const uint32_t u = __byte_perm(t0, t1, 0x5140);
        const uint32_t q = __byte_perm(t2, t3, 0x5140);
        o[0][w] ^= __byte_perm(u, q, 0x5410);
        if (NOUT > 1) o[NOUT > 1 ? 1 : 0][w] ^= __byte_perm(u, q, 0x7632);
        if (NOUT > 2) {
          const uint32_t u2 = __byte_perm(t0, t1, 0x7362);
          const uint32_t q2 = __byte_perm(t2, t3, 0x7362);
          o[NOUT > 2 ? 2 : 0][w] ^= __byte_perm(u2, q2, 0x5410);
          if (NOUT > 3) o[NOUT > 3 ? 3 : 0][w] ^= __byte_perm(u2, q2, 0x7632);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NOUT; ++j)
      if (off + 16 <= a.out_end[j])
        st16(seg(a.out_lo[j], a.out_hi[j], a.split, off), make_uint4(o[j][0], o[j][1], o[j][2], o[j][3]));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

// -------------------------------------------------------------- GF(2^16) ----
// Constant multiply c*w = c*(w & 0xff) ^ c*(w & 0xff00): two byte tables per
// input, entries pack the u16 products of outputs 0 (low half) and 1 (high).
template <int NOUT, int R, bool U>
__global__ void __launch_bounds__(1024) gf16_vec_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ uint32_t tab[];  // [nin][2][256][R]
  for (int e = threadIdx.x; e < a.nin * 512; e += blockDim.x) {
    const int i = e >> 9, h = (e >> 8) & 1, x = e & 255;
    const uint32_t v = h ? ((uint32_t)x << 8) : (uint32_t)x;
    uint32_t entry = gf16_mul(v, a.coef[0][i]);
    if (NOUT > 1) entry |= gf16_mul(v, a.coef[NOUT > 1 ? 1 : 0][i]) << 16;
    uint32_t* dst = tab + (size_t)e * R;
#pragma unroll
    for (int r = 0; r < R; ++r) dst[r] = entry;
  }
  __syncthreads();
  const uint32_t* tl = tab + (threadIdx.x & (R - 1));

  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += step) {
    const int64_t off = a.begin + (v << 4);
    uint32_t o[NOUT][4];
#pragma unroll
    for (int j = 0; j < NOUT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0u;
#pragma unroll 2
    for (int i = 0; i < a.nin; ++i) {
      const uint4 xv = U ? ldu16(a.in_lo[i] + off) : ld16(seg(a.in_lo[i], a.in_hi[i], a.split, off));
      const uint32_t* tlo = tl + (size_t)i * 512 * R;
      const uint32_t* thi = tlo + 256 * R;
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t x = xs[w];
        const uint32_t p0 = tlo[(x & 0xffu) * R] ^ thi[((x >> 8) & 0xffu) * R];
        const uint32_t p1 = tlo[((x >> 16) & 0xffu) * R] ^ thi[(x >> 24) * R];
        o[0][w] ^= __byte_perm(p0, p1, 0x5410);
        if (NOUT > 1) o[NOUT > 1 ? 1 : 0][w] ^= __byte_perm(p0, p1, 0x7632);
      }
    }
#pragma unroll
    for (int j = 0; j < NOUT; ++j)
      if (off + 16 <= a.out_end[j])
        st16(seg(a.out_lo[j], a.out_hi[j], a.split, off), make_uint4(o[j][0], o[j][1], o[j][2], o[j][3]));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

// ------------------------------------------------- XOR, unaligned inputs ----
// Inputs at any byte alignment (the bulk copies of the ring need 16-byte
// aligned sources): each thread XORs ldu16 windows of every input into an
// aligned 16-byte store of every output. Contiguous shards only.
__global__ void __launch_bounds__(256) xor_unaligned_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t nvec = (a.end - a.begin) >> 4;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += step) {
    const int64_t off = a.begin + (v << 4);
    uint4 acc = vzero();
    for (int i = 0; i < a.nin; ++i) acc = vxor(acc, ldu16(a.in_lo[i] + off));
    for (int o = 0; o < a.nout; ++o)
      if (off + 16 <= a.out_end[o]) st16(a.out_lo[o] + off, acc);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) linear_tail(a, a.begin + (nvec << 4));
}

// ---------------------------------------------------------------- scalar ----
// Misaligned layouts: one byte (XOR/GF8) or one u16 word (GF16) per thread.
__global__ void __launch_bounds__(256) linear_scalar_kernel(const LinearPass a) {
  grid_dep_wait();
  grid_dep_launch();
  const int sym = (a.field == Field::GF16) ? 2 : 1;
  const int64_t nsym = (a.end - a.begin) / sym;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < nsym; s += step) {
    const int64_t x = a.begin + s * sym;
    for (int j = 0; j < a.nout; ++j) {
      uint32_t acc = 0;
      for (int i = 0; i < a.nin; ++i) {
        const char* p = seg(a.in_lo[i], a.in_hi[i], a.split, x);
        if (a.field == Field::GF16) acc ^= gf16_mul(*reinterpret_cast<const uint16_t*>(p), a.coef[j][i]);
        else if (a.field == Field::GF8) acc ^= gf8_mul(*reinterpret_cast<const uint8_t*>(p), a.coef[j][i] & 0xffu);
        else acc ^= *reinterpret_cast<const uint8_t*>(p);
      }
      if (x + sym <= a.out_end[j]) {
        char* q = seg(a.out_lo[j], a.out_hi[j], a.split, x);
        if (a.field == Field::GF16) *reinterpret_cast<uint16_t*>(q) = (uint16_t)acc;
        else *reinterpret_cast<uint8_t*>(q) = (uint8_t)acc;
      }
    }
  }
}

bool pass_aligned(const LinearPass& a) {
  // a split at or past the end of the range (contiguous shards) never takes effect
  if ((a.begin & 15) || (a.split < a.end && (a.split & 15))) return false;
  for (int i = 0; i < a.nin; ++i)
    if (!aligned16(a.in_lo[i]) || !aligned16(a.in_hi[i])) return false;
  for (int j = 0; j < a.nout; ++j)
    if (!aligned16(a.out_lo[j]) || !aligned16(a.out_hi[j])) return false;
  return true;
}

template <typename K>
int occupancy_grid(K kernel, int threads, size_t smem, int64_t work_items) {
  LaunchCache& cache = launch_cache();
  int per_sm = cache.blocks_per_sm(kernel, threads, smem);
  if (per_sm < 1) per_sm = 1;
  int64_t grid = (int64_t)sm_count() * per_sm;
  const int64_t need = (work_items + threads - 1) / threads;
  if (need < grid) grid = need;
  return (int)(grid < 1 ? 1 : grid);
}

// Largest replication R (power of two <= 32) whose tables fit in `budget` bytes.
int pick_replicas(int64_t bytes_per_copy, int64_t budget) {
  int r = 32;
  while (r > 1 && bytes_per_copy * r > budget) r >>= 1;
  return r;
}

template <int NOUT, int R>
int launch_gf8(const LinearPass& a, cudaStream_t s) {
  const size_t smem = (size_t)a.nin * 256 * 4 * R;
  auto k = gf8_vec_kernel<NOUT, R>;
  const int threads = 1024;
  const int grid = occupancy_grid(k, threads, smem, (a.end - a.begin) >> 4);
  if (const cudaError_t lrc = launch_pdl(k, dim3((unsigned)(grid)), dim3(threads), smem, s, a))
    return launch_rc(lrc, "gf8_vec_kernel");
  return check_launch("gf8_vec_kernel");
}

template <int NOUT, int R, bool U>
int launch_gf16(const LinearPass& a, cudaStream_t s) {
  const size_t smem = (size_t)a.nin * 512 * 4 * R;
  auto k = gf16_vec_kernel<NOUT, R, U>;
  const int threads = 1024;
  const int grid = occupancy_grid(k, threads, smem, (a.end - a.begin) >> 4);
  if (const cudaError_t lrc = launch_pdl(k, dim3((unsigned)(grid)), dim3(threads), smem, s, a))
    return launch_rc(lrc, "gf16_vec_kernel");
  return check_launch("gf16_vec_kernel");
}

template <int NIN>
int launch_gf8_fixed(const LinearPass& a, cudaStream_t s) {
  constexpr int R = NIN <= 6 ? 32 : 16;
  const size_t smem = (size_t)NIN * 256 * 4 * (R + 1);
  bool flat = a.split >= a.end;
  for (int j = 0; j < a.nout; ++j) flat = flat && a.out_end[j] >= a.end;
  // Measured on B200: the flat form is 8 % faster with 4 and 5 inputs (RS(4,4),
  // RS(5,3) encodes) and 3 % slower with 6 (RS(6,2) decode); with 3 or fewer
  // ptxas gives it 32 registers and it spills. Only 4 and 5 use it.
  constexpr bool kFlat = NIN == 4 || NIN == 5;
  auto k = flat ? gf8_fixed_kernel<NIN, kFlat> : gf8_fixed_kernel<NIN, false>;
  const int threads = 1024;
  const int grid = occupancy_grid(k, threads, smem, (a.end - a.begin) >> 4);
  return launch_rc(launch_pdl(k, dim3(grid), dim3(threads), smem, s, a), "gf8_fixed_kernel");
}

template <int K, int M>
int launch_gf8_cauchy(const LinearPass& a, cudaStream_t s) {
  bool flat = a.split >= a.end;
  for (int j = 0; j < M; ++j) flat = flat && a.out_end[j] >= a.end;
  auto k = flat ? gf8_cauchy_kernel<K, M, true> : gf8_cauchy_kernel<K, M, false>;
  const int threads = 256;
  const int grid = occupancy_grid(k, threads, 0, ((((a.end - a.begin) >> 4) + 63) >> 6) * 32);
  return launch_rc(launch_pdl(k, dim3((unsigned)grid), dim3(threads), 0, s, a), "gf8_cauchy_kernel");
}

// The compile-time network when the pass's coefficients are the Cauchy
// generator's parity rows of RS(k, m) with 2 <= k, m <= 2, k + m <= 8; -1 when
// they are not. (Measured: with three or four parity rows the network costs
// more than the table kernel's lookups, which stay in use there.)
int try_gf8_cauchy(const LinearPass& a, cudaStream_t s) {
  for (int j = 0; j < a.nout; ++j)
    for (int i = 0; i < a.nin; ++i)
      if (a.coef[j][i] != cauchy_coef(a.nin, j, i)) return -1;
  switch (a.nin * 8 + a.nout) {
    case 2 * 8 + 1: return launch_gf8_cauchy<2, 1>(a, s);
    case 2 * 8 + 2: return launch_gf8_cauchy<2, 2>(a, s);
    case 3 * 8 + 1: return launch_gf8_cauchy<3, 1>(a, s);
    case 3 * 8 + 2: return launch_gf8_cauchy<3, 2>(a, s);
    case 4 * 8 + 1: return launch_gf8_cauchy<4, 1>(a, s);
    case 4 * 8 + 2: return launch_gf8_cauchy<4, 2>(a, s);
    case 5 * 8 + 1: return launch_gf8_cauchy<5, 1>(a, s);
    case 5 * 8 + 2: return launch_gf8_cauchy<5, 2>(a, s);
    case 6 * 8 + 1: return launch_gf8_cauchy<6, 1>(a, s);
    case 6 * 8 + 2: return launch_gf8_cauchy<6, 2>(a, s);
    case 7 * 8 + 1: return launch_gf8_cauchy<7, 1>(a, s);
    default: return -1;
  }
}

template <int NOUT>
int dispatch_gf8(const LinearPass& a, int r, cudaStream_t s) {
  switch (r) {
    case 32: return launch_gf8<NOUT, 32>(a, s);
    case 16: return launch_gf8<NOUT, 16>(a, s);
    case 8: return launch_gf8<NOUT, 8>(a, s);
    case 4: return launch_gf8<NOUT, 4>(a, s);
    case 2: return launch_gf8<NOUT, 2>(a, s);
    default: return launch_gf8<NOUT, 1>(a, s);
  }
}
template <int NOUT, bool U>
int dispatch_gf16(const LinearPass& a, int r, cudaStream_t s) {
  switch (r) {
    case 32: return launch_gf16<NOUT, 32, U>(a, s);
    case 16: return launch_gf16<NOUT, 16, U>(a, s);
    case 8: return launch_gf16<NOUT, 8, U>(a, s);
    case 4: return launch_gf16<NOUT, 4, U>(a, s);
    case 2: return launch_gf16<NOUT, 2, U>(a, s);
    default: return launch_gf16<NOUT, 1, U>(a, s);
  }
}

constexpr int64_t kTableBudget = 192 * 1024;

}  // namespace

namespace {
// XOR of byte c of every input (a row's head/tail bytes).
__device__ __forceinline__ char xor_byte(const RowCopyXor& a, int64_t c) {
  unsigned char v = 0;
  for (int r = 0; r < a.nin; ++r) v ^= static_cast<unsigned char>(a.in[r][c]);
  return static_cast<char>(v);
}

__global__ void __launch_bounds__(256) row_copy_xor_kernel(const RowCopyXor a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t ncopy = (a.copy_len + 15) >> 4;
  const uintptr_t first = reinterpret_cast<uintptr_t>(a.out0);
  const int64_t head = a.len > 0 ? (int64_t)(first & 15u) : 0;  // out0's offset in its aligned block
  char* base = reinterpret_cast<char*>(first - (uintptr_t)head);
  const int64_t nblk = a.len > 0 ? (head + a.len + 15) >> 4 : 0;
  const int64_t total = ncopy + nblk;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += step) {
    if (v < ncopy) {  // the copy: aligned vectors, bytes near the skipped range or the end one by one
      const int64_t o = v << 4;
      if (o + 16 <= a.copy_len && (o + 16 <= a.skip_lo || o >= a.skip_hi)) {
        st16(a.dst + o, ld16(a.src + o));
      } else {
        for (int b = 0; b < 16; ++b) {
          const int64_t x = o + b;
          if (x < a.copy_len && (x < a.skip_lo || x >= a.skip_hi)) a.dst[x] = a.src[x];
        }
      }
      continue;
    }
    // the XOR row: aligned 16-byte blocks of out0 (out1 shares its alignment),
    // inputs read through ldu16 windows; a partial first or last block bytewise
    const int64_t col = ((v - ncopy) << 4) - head;  // column of the block's first byte
    if (col >= 0 && col + 16 <= a.len) {
      uint4 x = vzero();
      for (int r = 0; r < a.nin; ++r) x = vxor(x, ldu16(a.in[r] + col));
      st16(base + head + col, x);
      if (a.out1 != nullptr) {
        if (col + 16 <= a.out1_len)
          st16(a.out1 + col, x);
        else
          for (int b = 0; b < 16 && col + b < a.out1_len; ++b) a.out1[col + b] = xor_byte(a, col + b);
      }
    } else {
      for (int b = 0; b < 16; ++b) {
        const int64_t c = col + b;
        if (c < 0 || c >= a.len) continue;
        const char val = xor_byte(a, c);
        a.out0[c] = val;
        if (a.out1 != nullptr && c < a.out1_len) a.out1[c] = val;
      }
    }
  }
}
}  // namespace

int run_row_copy_xor(const RowCopyXor& a, cudaStream_t s) {
  if (a.copy_len <= 0 && a.len <= 0) return GSEC_OK;
  if (a.nin < 1 || a.nin > kLinMaxIn || (a.copy_len > 0 && (!aligned16(a.src) || !aligned16(a.dst))) ||
      (a.out1 != nullptr && ((reinterpret_cast<uintptr_t>(a.out1) ^ reinterpret_cast<uintptr_t>(a.out0)) & 15u))) {
    set_error("row copy + XOR: bad inputs or alignment");
    return GSEC_EINVAL;
  }
  const int threads = 256;
  const int64_t work = ((a.copy_len + 15) >> 4) + ((a.len + 31) >> 4);
  const int grid = occupancy_grid(row_copy_xor_kernel, threads, 0, work);
  return launch_rc(launch_pdl(row_copy_xor_kernel, dim3((unsigned)grid), dim3(threads), 0, s, a),
                   "row_copy_xor_kernel");
}

unsigned linear_device_status(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_linear_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_linear_status, &z, sizeof(z));
  }
  return v;
}

namespace {
int run_scalar(const LinearPass& a, cudaStream_t s) {
  const int threads = 256;
  const int64_t nsym = (a.end - a.begin) / (a.field == Field::GF16 ? 2 : 1);
  const int grid = occupancy_grid(linear_scalar_kernel, threads, 0, nsym);
  if (const cudaError_t lrc = launch_pdl(linear_scalar_kernel, dim3((unsigned)(grid)), dim3(threads), 0, s, a))
    return launch_rc(lrc, "linear_scalar_kernel");
  return check_launch("linear_scalar_kernel");
}

// Layouts whose pointers are not 16-byte aligned (the reference's [rows, S]
// tensors with S not a multiple of 16 bytes). XOR and GF(2^16) passes over
// contiguous shards run with aligned stores and ldu16 input windows: outputs
// are grouped by their address mod 16, and each group's pass starts at the
// first offset where its outputs are aligned (the bytes before that go to the
// scalar kernel). Anything else keeps the scalar kernel.
int run_unaligned(const LinearPass& a, cudaStream_t s) {
  const bool contiguous = a.split >= a.end;
  const bool field_ok = a.field == Field::XOR || (a.field == Field::GF16 && (a.begin & 1) == 0);
  if (!contiguous || !field_ok || (a.end - a.begin) < 256) return run_scalar(a, s);
  bool done[kLinMaxOut] = {};
  for (int j = 0; j < a.nout; ++j) {
    if (done[j]) continue;
    const uintptr_t cls = reinterpret_cast<uintptr_t>(a.out_lo[j]) & 15u;
    LinearPass b = a;
    b.nout = 0;
    for (int q = j; q < a.nout; ++q) {
      if (done[q] || (reinterpret_cast<uintptr_t>(a.out_lo[q]) & 15u) != cls) continue;
      done[q] = true;
      b.out_lo[b.nout] = a.out_lo[q];
      b.out_hi[b.nout] = a.out_hi[q];
      b.out_end[b.nout] = a.out_end[q];
      for (int i = 0; i < a.nin; ++i) b.coef[b.nout][i] = a.coef[q][i];
      ++b.nout;
    }
    int64_t x = a.begin;
    while (((reinterpret_cast<uintptr_t>(b.out_lo[0]) + (uintptr_t)x) & 15u) && x < a.end) ++x;
    if (a.field == Field::GF16 && ((x - a.begin) & 1)) return run_scalar(a, s);  // odd byte output base
    if (x > a.begin) {  // the bytes before the first aligned output address
      LinearPass h = b;
      h.end = x < a.end ? x : a.end;
      const int rc = run_scalar(h, s);
      if (rc) return rc;
    }
    if (x >= a.end) continue;
    b.begin = x;
    int rc;
    if (a.field == Field::XOR) {
      const int threads = 256;
      const int grid = occupancy_grid(xor_unaligned_kernel, threads, 0, (b.end - b.begin) >> 4);
      if (const cudaError_t lrc = launch_pdl(xor_unaligned_kernel, dim3((unsigned)(grid)), dim3(threads), 0, s, b))
        return launch_rc(lrc, "xor_unaligned_kernel");
      rc = check_launch("xor_unaligned_kernel");
    } else {
      if (b.nout > 2) return run_scalar(a, s);
      const int r = pick_replicas((int64_t)b.nin * 512 * 4, kTableBudget);
      rc = b.nout == 1 ? dispatch_gf16<1, true>(b, r, s) : dispatch_gf16<2, true>(b, r, s);
    }
    if (rc) return rc;
  }
  return GSEC_OK;
}
}  // namespace

int run_linear(const LinearPass& a, cudaStream_t s) {
  if (a.end <= a.begin || a.nout == 0) return GSEC_OK;
  if (a.nin < 1 || a.nin > kLinMaxIn || a.nout < 0 || a.nout > kLinMaxOut) {
    set_error("linear pass: nin=%d nout=%d out of range", a.nin, a.nout);
    return GSEC_EINVAL;
  }
  if (!pass_aligned(a)) return run_unaligned(a, s);
  switch (a.field) {
    case Field::XOR:
      // measured: 2-3 inputs run best with 4 KiB stages and a 36 KiB ring, one
      // input with 4 KiB stages and the default ring, more inputs with 1 KiB stages
      if (a.nin <= GSEC_XOR_STREAM_MAXIN && !a.remote) {  // peer inputs: bulk copies over NVLink are faster
        const int threads = 256;
        const int64_t work = (((a.end - a.begin) >> 4) + 3) / 4;
        auto k = a.nin == 1 ? xor_stream_kernel<1> : (a.nin == 2 ? xor_stream_kernel<2> : xor_stream_kernel<3>);
        const int grid = occupancy_grid(k, threads, 0, work);
        return launch_rc(launch_pdl(k, dim3((unsigned)grid), dim3(threads), 0, s, a), "xor_stream_kernel");
      }
      return a.nin <= 3 ? launch_xor<4>(a, s, 2 * kLRingBytes) : launch_xor<1>(a, s, kLRingBytes);
    case Field::GF8: {
      if (a.nin >= 2 && a.nout >= 1) {
        const int rc = try_gf8_cauchy(a, s);
        if (rc >= 0) return rc;
      }
      switch (a.nin) {
        case 1: return launch_gf8_fixed<1>(a, s);
        case 2: return launch_gf8_fixed<2>(a, s);
        case 3: return launch_gf8_fixed<3>(a, s);
        case 4: return launch_gf8_fixed<4>(a, s);
        case 5: return launch_gf8_fixed<5>(a, s);
        case 6: return launch_gf8_fixed<6>(a, s);
        case 7: return launch_gf8_fixed<7>(a, s);
        case 8: return launch_gf8_fixed<8>(a, s);
        default: break;
      }
      const int r = pick_replicas((int64_t)a.nin * 256 * 4, kTableBudget);
      switch (a.nout) {
        case 1: return dispatch_gf8<1>(a, r, s);
        case 2: return dispatch_gf8<2>(a, r, s);
        case 3: return dispatch_gf8<3>(a, r, s);
        default: return dispatch_gf8<4>(a, r, s);
      }
    }
    case Field::GF16: {
      if (a.nout > 2) {
        set_error("GF16 pass has at most two outputs");
        return GSEC_EINVAL;
      }
      const int r = pick_replicas((int64_t)a.nin * 512 * 4, kTableBudget);
      return a.nout == 1 ? dispatch_gf16<1, false>(a, r, s) : dispatch_gf16<2, false>(a, r, s);
    }
  }
  return GSEC_EINVAL;
}

}  // namespace gsec
