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

__device__ __forceinline__ int64_t mod_s(int64_t x, int64_t S) {
  int64_t r = x % S;
  return r < 0 ? r + S : r;
}

// excl[r]: the Q position whose row-r term is skipped, or -1.
__global__ void __launch_bounds__(256) rdpref_parity_kernel(RdpRefParityArgs a) {
  const int64_t S = a.S;
  const int64_t nvec = (S + 7) >> 3;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  uint16_t* prow = a.rows + (int64_t)a.nd * a.pitch;
  uint16_t* qrow = a.rows + (int64_t)(a.nd + 1) * a.pitch;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += step) {
    const int64_t d0 = t << 3;
    const bool interior = a.vec_ok && d0 >= (int64_t)(a.nd - 1) && d0 + 8 <= S;
    if (interior) {
      uint4 p = vzero(), q = vzero();
      for (int rb = 0; rb < a.nd; rb += 8) {
        const int64_t vq = rb >> 3;  // whole-vector shift of this group of rows
#pragma unroll
        for (int w = 0; w < 8; ++w) {  // word shift; a literal after unrolling
          const int r = rb + w;
          if (r >= a.nd) break;
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
      const int64_t dend = d0 + 8 < S ? d0 + 8 : S;
      for (int64_t d = d0; d < dend; ++d) {
        uint16_t pacc = 0, qacc = 0;
        for (int r = 0; r < a.nd; ++r) {
          const uint16_t* row = a.rows + (int64_t)r * a.pitch;
          pacc ^= row[d];
          const int64_t c = mod_s(d - r, S);
          if (a.excl[r] == d) continue;  // c == star_r
          qacc ^= row[c];
        }
        prow[d] = pacc;
        qrow[d] = qacc;
      }
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
  const int64_t nvec = (S + 7) >> 3;
  const int threads = 256;
  int64_t grid = (nvec + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  rdpref_parity_kernel<<<(int)grid, threads, 0, s>>>(a);
  return check_launch("rdpref_parity_kernel");
}

}  // namespace gsec
