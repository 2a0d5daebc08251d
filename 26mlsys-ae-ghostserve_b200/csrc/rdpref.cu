// rdpref.cu — the reference's row/diagonal parity over u16 words, reproduced
// bit for bit (benchmark/rdp/kernel.cu:76-107, bench_ghostserve_rdp.py:121-150):
//   P[c] = XOR_{r<nd} D[r][c]
//   Q[d] = XOR_{r<nd} D[r][(d - r) mod S], skipping the cell where
//          (d - r) mod S == star_r, star_r = (star_base + r) % S (C remainder;
//          a negative star_r never matches).
// Q reads each data row shifted right by r words with wrap-around at S.
//
// Vector path: a thread owns 8 consecutive words [d0, d0+8) of P and Q.  For row
// r the window [d0 - r, d0 - r + 8) straddles two aligned 16-byte vectors; it is
// assembled with byte permutes whose selectors are compile-time constants
// because the row loop is unrolled (shift = r mod 8 words, vector offset = r/8).
// The vector at d0 also feeds P.  Threads whose window wraps (d0 < nd-1) or runs
// past S, and layouts that are not 16-byte aligned, use the scalar path, which is
// the reference formula word by word.
#include "common.cuh"
#include "rdpref.cuh"

namespace gsec {
namespace {

constexpr int kRefMaxNd = 32;

__device__ __forceinline__ uint4 ld16c(const uint16_t* p) {  // cached: neighbours reuse it
  return *reinterpret_cast<const uint4*>(p);
}

// 8 words starting `w` words into the 16-word concatenation [lo | hi].
template <int W>
__device__ __forceinline__ uint4 window(uint4 lo, uint4 hi) {
  const uint32_t e[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  uint32_t o[4];
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    if ((W & 1) == 0) {
      o[l] = e[(W >> 1) + l];
    } else {
      const int m = (W >> 1) + l;
      o[l] = __byte_perm(e[m], e[m + 1 < 8 ? m + 1 : 7], 0x5432);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint4 window_rt(int w, uint4 lo, uint4 hi) {
  switch (w) {
    case 0: return window<0>(lo, hi);
    case 1: return window<1>(lo, hi);
    case 2: return window<2>(lo, hi);
    case 3: return window<3>(lo, hi);
    case 4: return window<4>(lo, hi);
    case 5: return window<5>(lo, hi);
    case 6: return window<6>(lo, hi);
    default: return window<7>(lo, hi);
  }
}

// Clear word lane i (0..7) of a vector.
__device__ __forceinline__ uint4 clear_lane(uint4 v, int i) {
  const uint32_t keep = (i & 1) ? 0x0000ffffu : 0xffff0000u;
  switch (i >> 1) {
    case 0: v.x &= keep; break;
    case 1: v.y &= keep; break;
    case 2: v.z &= keep; break;
    default: v.w &= keep; break;
  }
  return v;
}

// (x mod S) for x > -nd: one add unless S < nd (tiny shards), then a modulo.
__device__ __forceinline__ int64_t wrap_s(int64_t x, int64_t S) {
  if (x >= 0) return x;
  x += S;
  return x >= 0 ? x : ((x % S) + S) % S;
}

// excl[r]: the Q position whose row-r term is skipped, or -1.
// ND > 0: the row count as a compile-time constant, so every row's loads are
// independent straight-line code (all in flight at once); ND = 0: any count.
template <int ND>
__global__ void __launch_bounds__(256) rdpref_parity_kernel(RdpRefParityArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int nd = ND > 0 ? ND : a.nd;
  const int64_t S = a.S;
  const int64_t nvec = (S + 7) >> 3;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  uint16_t* prow = a.rows + (int64_t)nd * a.pitch;
  uint16_t* qrow = a.rows + (int64_t)(nd + 1) * a.pitch;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += step) {
    const int64_t d0 = t << 3;
    const bool interior = a.vec_ok && d0 >= (int64_t)(nd - 1) && d0 + 8 <= S;
    if (interior) {
      uint4 p = vzero(), q = vzero();
#pragma unroll
      for (int rb = 0; rb < (ND > 0 ? ND : kRefMaxNd); rb += 8) {
        if (ND == 0 && rb >= nd) break;
        const int64_t vq = rb >> 3;  // whole-vector shift of this group of rows
#pragma unroll
        for (int w = 0; w < 8; ++w) {  // word shift; a literal after unrolling
          const int r = rb + w;
          if (r >= nd) break;
          const uint16_t* row = a.rows + (int64_t)r * a.pitch;
          const uint4 at_d0 = ld16c(row + d0);
          p = vxor(p, at_d0);
          const uint4 hi = vq == 0 ? at_d0 : ld16c(row + d0 - 8 * vq);
          uint4 win = hi;
          if (w != 0) win = window_rt(8 - w, ld16c(row + d0 - 8 * vq - 8), hi);
          const int64_t ex = a.excl[r];
          if (ex >= d0 && ex < d0 + 8) win = clear_lane(win, (int)(ex - d0));
          q = vxor(q, win);
        }
      }
      *reinterpret_cast<uint4*>(prow + d0) = p;
      *reinterpret_cast<uint4*>(qrow + d0) = q;
    } else {
      // the wrapping head (d0 < nd - 1) and the partial tail: word by word, with
      // every row's two loads independent of each other
      const int64_t dend = d0 + 8 < S ? d0 + 8 : S;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int64_t d = d0 + e;
        if (d >= dend) break;
        uint16_t pacc = 0, qacc = 0;
#pragma unroll
        for (int r = 0; r < (ND > 0 ? ND : kRefMaxNd); ++r) {
          if (ND == 0 && r >= nd) break;
          const uint16_t* row = a.rows + (int64_t)r * a.pitch;
          const int64_t c = wrap_s(d - r, S);
          const uint16_t pw = row[d], qw = row[c];
          pacc ^= pw;
          qacc ^= a.excl[r] == d ? (uint16_t)0 : qw;  // c == star_r: skipped
        }
        prow[d] = pacc;
        qrow[d] = qacc;
      }
    }
  }
}

// Any row alignment (pitch not a multiple of 8 words, or an unaligned base):
// P and Q are written with aligned 16-byte stores of their own rows (work item
// g < np covers a P vector, the rest Q vectors); every row is read through
// ldu16 windows (P at d0, Q at d0 - r). Unaligned heads, the wrapping start of
// Q (d0 < nd - 1) and partial tails use the scalar formula.
__device__ __forceinline__ void ref_words(const RdpRefParityArgs& a, int64_t d, uint16_t* pw, uint16_t* qw) {
  uint16_t pacc = 0, qacc = 0;
#pragma unroll
  for (int r = 0; r < kRefMaxNd; ++r) {  // loads independent of each other
    if (r >= a.nd) break;
    const uint16_t* row = a.rows + (int64_t)r * a.pitch;
    const int64_t c = wrap_s(d - r, a.S);
    const uint16_t p = row[d], q = row[c];
    pacc ^= p;
    qacc ^= a.excl[r] == d ? (uint16_t)0 : q;
  }
  if (pw) *pw = pacc;
  if (qw) *qw = qacc;
}

__global__ void __launch_bounds__(256) rdpref_parity_any(RdpRefParityArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t S = a.S;
  const int64_t slots = (S >> 3) + 2;
  uint16_t* prow = a.rows + (int64_t)a.nd * a.pitch;
  uint16_t* qrow = a.rows + (int64_t)(a.nd + 1) * a.pitch;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < 2 * slots; g += (int64_t)gridDim.x * blockDim.x) {
    const bool isp = g < slots;
    uint16_t* out = isp ? prow : qrow;
    const int64_t j = isp ? g : g - slots;
    int64_t h = ((16 - (int64_t)(reinterpret_cast<uintptr_t>(out) & 15u)) & 15) >> 1;
    if (h > S) h = S;
    const int64_t d0 = j == 0 ? 0 : h + (j - 1) * 8;
    const int64_t d1 = j == 0 ? h : (d0 + 8 < S ? d0 + 8 : S);
    if (d0 >= d1) continue;
    const bool full = d1 - d0 == 8;
    if (isp && full) {
      uint4 acc = vzero();
      for (int r = 0; r < a.nd; ++r) acc = vxor(acc, ldu16(a.rows + (int64_t)r * a.pitch + d0));
      *reinterpret_cast<uint4*>(out + d0) = acc;
    } else if (!isp && full && d0 >= (int64_t)(a.nd - 1)) {
      uint4 acc = vzero();
      for (int r = 0; r < a.nd; ++r) {
        uint4 win = ldu16(a.rows + (int64_t)r * a.pitch + d0 - r);
        const int64_t ex = a.excl[r];
        if (ex >= d0 && ex < d0 + 8) win = clear_lane(win, (int)(ex - d0));
        acc = vxor(acc, win);
      }
      *reinterpret_cast<uint4*>(out + d0) = acc;
    } else {
      for (int64_t d = d0; d < d1; ++d) ref_words(a, d, isp ? out + d : nullptr, isp ? nullptr : out + d);
    }
  }
}

}  // namespace

int rdpref_parity(uint16_t* rows, int64_t pitch, int nd, int64_t S, int star_base, cudaStream_t s) {
  GSEC_REQUIRE(rows != nullptr, "rows is null");
  GSEC_REQUIRE(nd >= 1 && nd <= kRefMaxNd, "nd=%d must be in [1, %d]", nd, kRefMaxNd);
  GSEC_REQUIRE(S >= 1, "S=%lld must be positive", (long long)S);
  GSEC_REQUIRE(pitch >= S, "row pitch %lld < S %lld", (long long)pitch, (long long)S);
  RdpRefParityArgs a{};
  a.rows = rows;
  a.pitch = pitch;
  a.nd = nd;
  a.S = S;
  for (int r = 0; r < nd; ++r) {
    // star_r = (star_base + r) % S with C semantics, as in the reference (int arithmetic).
    const long long sr = ((long long)star_base + r) % S;
    a.excl[r] = sr < 0 ? -1 : (int64_t)((sr + r) % S);
  }
  a.vec_ok = aligned16(rows) && (pitch % 8 == 0);
  const int threads = 256;
  if (!a.vec_ok) {
    int64_t grid = (2 * ((S >> 3) + 2) + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 8;
    grid = grid > cap ? cap : (grid < 1 ? 1 : grid);
    if (const cudaError_t lrc = launch_pdl(rdpref_parity_any, dim3((unsigned)((int)grid)), dim3(threads), 0, s, a))
      return launch_rc(lrc, "rdpref_parity_any");
    return check_launch("rdpref_parity_any");
  }
  const int64_t nvec = (S + 7) >> 3;
  int64_t grid = (nvec + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  switch (nd) {
    case 2:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<2>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 3:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<3>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 4:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<4>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 5:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<5>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 6:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<6>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 7:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<7>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    case 8:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<8>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
    default:
      if (const cudaError_t lrc = launch_pdl(rdpref_parity_kernel<0>, dim3((unsigned)((int)grid)), dim3(threads), 0,
                                             s, a))
        return launch_rc(lrc, "rdpref_parity_kernel");
      break;
  }
  return check_launch("rdpref_parity_kernel");
}

}  // namespace gsec
