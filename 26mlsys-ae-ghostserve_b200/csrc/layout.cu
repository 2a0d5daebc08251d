// layout.cu — moves between the KV tensors and shard rows.
//
// The reference packs K and V into a separate byte/word stream, pads it, and
// then copies the stream into shard rows (benchmark/xor/main.py:80-93,
// benchmark/rs/main.py:90-110, benchmark/rdp/kernel.cu:32-72) — three passes.
// Here one kernel reads K and V where they lie and writes the rows:
//   rows_pack   : stream = K ++ V (byte order), row r = stream[r*row_bytes ...],
//                 zero past the stream end
//   rows_unpack : the inverse
//   bhtd_pack   : the reference RDP stream is token-major ([T, B*H*D] per
//                 tensor, benchmark/rdp/main.py:66-67); this reads [B,H,T,D]
//                 and applies the permutation on the fly
//   bhtd_unpack : the inverse (benchmark/rdp/kernel.cu:305-345 + main.py:121-124)
// Vector paths move 16 bytes per thread when every address involved is
// 16-byte aligned; otherwise one byte (or u16 word) per thread.
#include "common.cuh"
#include "layout.cuh"
#include "pipe.cuh"

namespace gsec {
namespace {

__device__ __forceinline__ uint4 ldv(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void stv(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

int grid_cap(int64_t items, int threads) {
  int64_t g = (items + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

// ----------------------------------------------------------- rows <-> stream
__global__ void rows_pack_vec(const char* s0, int64_t len0, const char* s1, int64_t len1, char* rows,
                              int64_t pitch, int64_t row_bytes, int nrows) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t vpr = row_bytes >> 4;  // row_bytes is a multiple of 16 here
  const int64_t total = vpr * nrows;
  const int64_t stream = len0 + len1;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / vpr, x = (v - r * vpr) << 4;
    const int64_t i = r * row_bytes + x;
    char* dst = rows + r * pitch + x;
    if (i + 16 <= len0) {
      stv(dst, ldv(s0 + i));
    } else if (i >= len0 && i + 16 <= stream) {
      stv(dst, ldv(s1 + (i - len0)));
    } else if (i >= stream) {
      stv(dst, vzero());
    } else {
      for (int b = 0; b < 16; ++b) {
        const int64_t j = i + b;
        dst[b] = j < len0 ? s0[j] : (j < stream ? s1[j - len0] : (char)0);
      }
    }
  }
}

// Any alignment: every row is written with aligned 16-byte stores (its first
// bytes up to the first aligned address, and its last partial vector, byte by
// byte); the stream is read with ldu16 windows.
__device__ __forceinline__ char stream_byte(const char* s0, int64_t len0, const char* s1, int64_t stream,
                                            int64_t j) {
  return j < len0 ? s0[j] : (j < stream ? s1[j - len0] : (char)0);
}

__global__ void rows_pack_any(const char* s0, int64_t len0, const char* s1, int64_t len1, char* rows,
                              int64_t pitch, int64_t row_bytes, int nrows) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t slots = (row_bytes >> 4) + 2;  // head + whole vectors + tail of a row
  const int64_t total = slots * nrows;
  const int64_t stream = len0 + len1;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = g / slots, j = g - r * slots;
    char* base = rows + r * pitch;
    int64_t h = (16 - (int64_t)(reinterpret_cast<uintptr_t>(base) & 15u)) & 15;
    if (h > row_bytes) h = row_bytes;
    const int64_t x0 = j == 0 ? 0 : h + (j - 1) * 16;
    const int64_t x1 = j == 0 ? h : (x0 + 16 < row_bytes ? x0 + 16 : row_bytes);
    if (x0 >= x1) continue;
    const int64_t i = r * row_bytes + x0;  // stream offset of base[x0]
    if (x1 - x0 == 16 && i + 16 <= len0) {
      stv(base + x0, ldu16(s0 + i));
    } else if (x1 - x0 == 16 && i >= len0 && i + 16 <= stream) {
      stv(base + x0, ldu16(s1 + (i - len0)));
    } else if (x1 - x0 == 16 && i >= stream) {
      stv(base + x0, vzero());
    } else {
      for (int64_t x = x0; x < x1; ++x) base[x] = stream_byte(s0, len0, s1, stream, r * row_bytes + x);
    }
  }
}

__global__ void rows_unpack_vec(const char* rows, int64_t pitch, int64_t row_bytes, char* d0, int64_t len0,
                                char* d1, int64_t len1) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stream = len0 + len1;
  const int64_t total = (stream + 15) >> 4;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v << 4;
    const int64_t r = i / row_bytes, x = i - r * row_bytes;
    const char* src = rows + r * pitch + x;
    if (i + 16 <= len0) {
      stv(d0 + i, ldv(src));
    } else if (i >= len0 && i + 16 <= stream) {
      stv(d1 + (i - len0), ldv(src));
    } else {
      for (int b = 0; b < 16 && i + b < stream; ++b) {
        const int64_t j = i + b;
        if (j < len0) d0[j] = src[b];
        else d1[j - len0] = src[b];
      }
    }
  }
}

// Any alignment: each destination (d0, then d1) is written with aligned
// 16-byte stores, its unaligned head and last partial vector byte by byte; a
// vector whose 16 source bytes lie in one row is read with an ldu16 window.
__global__ void rows_unpack_any(const char* rows, int64_t pitch, int64_t row_bytes, char* d0, int64_t len0,
                                char* d1, int64_t len1) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t na = (len0 >> 4) + 2, nb = (len1 >> 4) + 2;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < na + nb; g += (int64_t)gridDim.x * blockDim.x) {
    const bool first = g < na;
    char* dst = first ? d0 : d1;
    const int64_t len = first ? len0 : len1, soff = first ? 0 : len0, j = first ? g : g - na;
    if (len == 0) continue;
    int64_t h = (16 - (int64_t)(reinterpret_cast<uintptr_t>(dst) & 15u)) & 15;
    if (h > len) h = len;
    const int64_t x0 = j == 0 ? 0 : h + (j - 1) * 16;
    const int64_t x1 = j == 0 ? h : (x0 + 16 < len ? x0 + 16 : len);
    if (x0 >= x1) continue;
    const int64_t i = soff + x0;  // stream offset of dst[x0]
    const int64_t r = i / row_bytes, x = i - r * row_bytes;
    if (x1 - x0 == 16 && x + 16 <= row_bytes) {
      stv(dst + x0, ldu16(rows + r * pitch + x));
    } else {
      for (int64_t b = x0; b < x1; ++b) {
        const int64_t ii = soff + b, rr = ii / row_bytes;
        dst[b] = rows[rr * pitch + (ii - rr * row_bytes)];
      }
    }
  }
}

// ------------------------------------------------------ [B,H,T,D] <-> rows --
// Token-major stream index i (words): tensor = i / (T*n), j = i % (T*n),
// t = j / n, c = j % n, bh = c / D, d = c % D; source word (bh*T + t)*D + d.
struct Perm {
  int64_t T, D, n, Tn;
  bool small;                  // every stream/source index and row slot fits 32 bits: fast division
  FastDiv fn, fD, fT, fslots;  // by n, D, T and the row-slot count of the *_any kernels
};

Perm make_perm(int64_t B, int64_t H, int64_t T, int64_t D, int64_t slots) {
  Perm p{T, D, B * H * D, T * B * H * D, false, FastDiv(), FastDiv(), FastDiv(), FastDiv()};
  p.small = 2 * p.Tn + 64 < (1ll << 31) && slots < (1ll << 31);
  if (p.small) {
    p.fn = FastDiv((uint32_t)p.n);
    p.fD = FastDiv((uint32_t)D);
    p.fT = FastDiv((uint32_t)T);
    p.fslots = FastDiv((uint32_t)(slots > 0 ? slots : 1));
  }
  return p;
}

__device__ __forceinline__ int64_t perm_src(const Perm& p, int64_t j) {
  if (p.small) {
    const uint32_t jj = (uint32_t)j, t = p.fn.div(jj), c = jj - t * (uint32_t)p.n;
    const uint32_t bh = p.fD.div(c), d = c - bh * (uint32_t)p.D;
    return (int64_t)((bh * (uint32_t)p.T + t) * (uint32_t)p.D + d);
  }
  const int64_t t = j / p.n, c = j - t * p.n;
  const int64_t bh = c / p.D, d = c - bh * p.D;
  return (bh * p.T + t) * p.D + d;
}

// (word d within its run of D, and the run's token-major stream index) helpers
__device__ __forceinline__ int64_t perm_d(const Perm& p, int64_t j) {
  if (p.small) {
    const uint32_t jj = (uint32_t)j, t = p.fn.div(jj), c = jj - t * (uint32_t)p.n;
    return (int64_t)(c - p.fD.div(c) * (uint32_t)p.D);
  }
  return (j % p.n) % p.D;
}

// Vector path needs D % 8 == 0, S % 8 == 0, aligned rows/pitch/tensors: then a
// group of 8 stream words maps to 8 consecutive source words.
__global__ void bhtd_pack_kernel(const uint16_t* k, const uint16_t* v, Perm p, uint16_t* rows, int64_t pitch,
                                 int64_t S, int nd, bool vec) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t groups = (S + 7) >> 3;
  const int64_t total = groups * nd;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = g / groups, c0 = (g - r * groups) << 3;
    const int64_t i0 = r * S + c0;
    uint16_t* dst = rows + r * pitch + c0;
    if (vec && c0 + 8 <= S && i0 + 8 <= 2 * p.Tn) {
      const uint16_t* src = i0 < p.Tn ? k + perm_src(p, i0) : v + perm_src(p, i0 - p.Tn);
      stv(dst, ldv(src));
    } else {
      for (int b = 0; b < 8 && c0 + b < S; ++b) {
        const int64_t i = i0 + b;
        dst[b] = i < p.Tn ? k[perm_src(p, i)] : (i < 2 * p.Tn ? v[perm_src(p, i - p.Tn)] : (uint16_t)0);
      }
    }
  }
}

__global__ void bhtd_unpack_kernel(const uint16_t* rows, int64_t pitch, int64_t S, Perm p, uint16_t* k,
                                   uint16_t* v, bool vec) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t total = (2 * p.Tn + 7) >> 3;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = g << 3;
    const int64_t r = i0 / S, c0 = i0 - r * S;
    if (vec && c0 + 8 <= S && i0 + 8 <= 2 * p.Tn) {
      const uint4 val = ldv(rows + r * pitch + c0);
      uint16_t* dst = i0 < p.Tn ? k + perm_src(p, i0) : v + perm_src(p, i0 - p.Tn);
      stv(dst, val);
    } else {
      for (int b = 0; b < 8 && i0 + b < 2 * p.Tn; ++b) {
        const int64_t i = i0 + b;
        const int64_t rr = i / S, cc = i - rr * S;
        const uint16_t w = rows[rr * pitch + cc];
        if (i < p.Tn) k[perm_src(p, i)] = w;
        else v[perm_src(p, i - p.Tn)] = w;
      }
    }
  }
}

// Any alignment (D, S, pitch or a tensor not multiples of 8 words / 16 bytes):
// rows are written with aligned 16-byte stores (unaligned head and last partial
// vector word by word); 8 stream words that are 8 consecutive source words
// (same token, same [b,h], d + 8 <= D) are read with one ldu16 window.
__device__ __forceinline__ uint16_t bhtd_word(const uint16_t* k, const uint16_t* v, const Perm& p, int64_t i) {
  return i < p.Tn ? k[perm_src(p, i)] : (i < 2 * p.Tn ? v[perm_src(p, i - p.Tn)] : (uint16_t)0);
}

__global__ void bhtd_pack_any(const uint16_t* k, const uint16_t* v, Perm p, uint16_t* rows, int64_t pitch,
                              int64_t S, int nd) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t slots = (S >> 3) + 2;
  const int64_t total = slots * nd;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = p.small ? (int64_t)p.fslots.div((uint32_t)g) : g / slots, j = g - r * slots;
    uint16_t* base = rows + r * pitch;
    int64_t h = ((16 - (int64_t)(reinterpret_cast<uintptr_t>(base) & 15u)) & 15) >> 1;  // words
    if (h > S) h = S;
    const int64_t c0 = j == 0 ? 0 : h + (j - 1) * 8;
    const int64_t c1 = j == 0 ? h : (c0 + 8 < S ? c0 + 8 : S);
    if (c0 >= c1) continue;
    const int64_t i0 = r * S + c0;
    bool done = false;
    if (c1 - c0 == 8 && (reinterpret_cast<uintptr_t>(base + c0) & 15u) == 0) {
      if (i0 >= 2 * p.Tn) {
        stv(base + c0, vzero());
        done = true;
      } else if (i0 + 8 <= p.Tn || (i0 >= p.Tn && i0 + 8 <= 2 * p.Tn)) {
        const uint16_t* src = i0 < p.Tn ? k : v;
        const int64_t jj = i0 < p.Tn ? i0 : i0 - p.Tn;
        const int64_t d = perm_d(p, jj);
        if (d + 8 <= p.D) {
          stv(base + c0, ldu16(src + perm_src(p, jj)));
          done = true;
        } else if (p.D >= 8) {
          // the 8 words straddle two runs of D: the first kk words end run A, the
          // rest start run B; B is read as a window starting kk words early and
          // its first kk words are replaced by A's
          const int kk = (int)(p.D - d);
          const uint4 a = ldu16(src + perm_src(p, jj));
          const uint4 b = ldu16(src + perm_src(p, jj + kk) - kk);
          const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
          uint32_t o[4];
#pragma unroll
          for (int l = 0; l < 4; ++l) {  // words 2l, 2l+1 of the result
            const uint32_t m = (2 * l + 1 < kk) ? 0xffffffffu : (2 * l < kk ? 0x0000ffffu : 0u);
            o[l] = (av[l] & m) | (bv[l] & ~m);
          }
          stv(base + c0, make_uint4(o[0], o[1], o[2], o[3]));
          done = true;
        }
      }
    }
    if (!done)
      for (int64_t c = c0; c < c1; ++c) base[c] = bhtd_word(k, v, p, r * S + c);
  }
}

// Inverse: the K and V tensors are written in [B,H,T,D] order with aligned
// 16-byte stores; 8 destination words in one [b,h,t] run of D come from 8
// consecutive stream words, read with one ldu16 window when they lie in one row.
__global__ void bhtd_unpack_any(const uint16_t* rows, int64_t pitch, int64_t S, Perm p, uint16_t* k,
                                uint16_t* v) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t per = (p.Tn >> 3) + 2;  // slots of one tensor
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < 2 * per; g += (int64_t)gridDim.x * blockDim.x) {
    const bool isk = g < per;
    uint16_t* dst = isk ? k : v;
    const int64_t j = isk ? g : g - per, toff = isk ? 0 : p.Tn;
    int64_t h = ((16 - (int64_t)(reinterpret_cast<uintptr_t>(dst) & 15u)) & 15) >> 1;
    if (h > p.Tn) h = p.Tn;
    const int64_t w0 = j == 0 ? 0 : h + (j - 1) * 8;
    const int64_t w1 = j == 0 ? h : (w0 + 8 < p.Tn ? w0 + 8 : p.Tn);
    if (w0 >= w1) continue;
    // destination word w = ((bh * T + t) * D + d)  ->  stream word t * n + bh * D + d
    int64_t d, t, bh;
    if (p.small) {
      const uint32_t bt = p.fD.div((uint32_t)w0), b2 = p.fT.div(bt);
      d = (int64_t)((uint32_t)w0 - bt * (uint32_t)p.D);
      t = (int64_t)(bt - b2 * (uint32_t)p.T);
      bh = (int64_t)b2;
    } else {
      d = w0 % p.D;
      t = (w0 / p.D) % p.T;
      bh = (w0 / p.D) / p.T;
    }
    const int64_t i = toff + t * p.n + bh * p.D + d;
    const int64_t r = i / S, x = i - r * S;
    if (w1 - w0 == 8 && d + 8 <= p.D && x + 8 <= S && (reinterpret_cast<uintptr_t>(dst + w0) & 15u) == 0) {
      stv(dst + w0, ldu16(rows + r * pitch + x));
    } else {
      for (int64_t w = w0; w < w1; ++w) {
        const int64_t dd = w % p.D, b2 = w / p.D, tt = b2 % p.T, bb = b2 / p.T;
        const int64_t ii = toff + tt * p.n + bb * p.D + dd, rr = ii / S;
        dst[w] = rows[rr * pitch + (ii - rr * S)];
      }
    }
  }
}

}  // namespace

int rows_pack(const void* s0, int64_t len0, const void* s1, int64_t len1, void* rows, int64_t pitch,
              int64_t row_bytes, int nrows, cudaStream_t s) {
  GSEC_REQUIRE(rows != nullptr && nrows >= 1 && row_bytes >= 1, "rows_pack: bad rows");
  GSEC_REQUIRE(pitch >= row_bytes, "rows_pack: pitch < row_bytes");
  GSEC_REQUIRE(len0 >= 0 && len1 >= 0 && (len0 == 0 || s0) && (len1 == 0 || s1), "rows_pack: bad stream");
  GSEC_REQUIRE(len0 + len1 <= row_bytes * nrows, "rows_pack: stream longer than the rows");
  const char* a = static_cast<const char*>(s0);
  const char* b = static_cast<const char*>(s1);
  const bool vec = (row_bytes % 16 == 0) && (pitch % 16 == 0) && (len0 % 16 == 0) && aligned16(rows) &&
                   (len0 == 0 || aligned16(a)) && (len1 == 0 || aligned16(b));
  const int threads = 256;
  if (vec) {
    if (const cudaError_t lrc = launch_pdl(rows_pack_vec,
                                           dim3((unsigned)(grid_cap((row_bytes >> 4) * nrows, threads))),
                                           dim3(threads), 0, s, a, len0, b, len1, static_cast<char*>(rows), pitch,
                                           row_bytes, nrows))
      return launch_rc(lrc, "rows_pack_vec");
  } else {
    if (const cudaError_t lrc = launch_pdl(rows_pack_any,
                                           dim3((unsigned)(grid_cap(((row_bytes >> 4) + 2) * nrows, threads))),
                                           dim3(threads), 0, s, a, len0, b, len1, static_cast<char*>(rows), pitch,
                                           row_bytes, nrows))
      return launch_rc(lrc, "rows_pack_any");
  }
  return check_launch("rows_pack");
}

int rows_unpack(const void* rows, int64_t pitch, int64_t row_bytes, int nrows, void* d0, int64_t len0, void* d1,
                int64_t len1, cudaStream_t s) {
  GSEC_REQUIRE(rows != nullptr && nrows >= 1 && row_bytes >= 1, "rows_unpack: bad rows");
  GSEC_REQUIRE(pitch >= row_bytes, "rows_unpack: pitch < row_bytes");
  GSEC_REQUIRE(len0 >= 0 && len1 >= 0 && (len0 == 0 || d0) && (len1 == 0 || d1), "rows_unpack: bad outputs");
  GSEC_REQUIRE(len0 + len1 <= row_bytes * nrows, "rows_unpack: stream longer than the rows");
  char* a = static_cast<char*>(d0);
  char* b = static_cast<char*>(d1);
  const bool vec = (row_bytes % 16 == 0) && (pitch % 16 == 0) && (len0 % 16 == 0) && aligned16(rows) &&
                   (len0 == 0 || aligned16(a)) && (len1 == 0 || aligned16(b));
  const int threads = 256;
  if (vec) {
    if (const cudaError_t lrc = launch_pdl(rows_unpack_vec,
                                           dim3((unsigned)(grid_cap((len0 + len1 + 15) >> 4, threads))),
                                           dim3(threads), 0, s, static_cast<const char*>(rows), pitch, row_bytes, a,
                                           len0, b, len1))
      return launch_rc(lrc, "rows_unpack_vec");
  } else {
    if (const cudaError_t lrc = launch_pdl(rows_unpack_any,
                                           dim3((unsigned)(grid_cap((len0 >> 4) + (len1 >> 4) + 4, threads))),
                                           dim3(threads), 0, s, static_cast<const char*>(rows), pitch, row_bytes, a,
                                           len0, b, len1))
      return launch_rc(lrc, "rows_unpack_any");
  }
  return check_launch("rows_unpack");
}

int bhtd_pack(const uint16_t* k, const uint16_t* v, int64_t B, int64_t H, int64_t T, int64_t D, uint16_t* rows,
              int64_t pitch, int nd, int64_t S, cudaStream_t s) {
  GSEC_REQUIRE(k && v && rows && B >= 1 && H >= 1 && T >= 1 && D >= 1 && nd >= 1, "bhtd_pack: bad args");
  Perm p = make_perm(B, H, T, D, (S >> 3) + 2);
  if (((S >> 3) + 2) * nd >= (1ll << 31)) p.small = false;  // slot indices past 32 bits
  GSEC_REQUIRE(S * nd >= 2 * p.Tn && pitch >= S, "bhtd_pack: rows too small");
  const bool vec = (D % 8 == 0) && (S % 8 == 0) && (pitch % 8 == 0) && aligned16(k) && aligned16(v) && aligned16(rows);
  const int threads = 256;
  if (!vec) {
    if (const cudaError_t lrc = launch_pdl(bhtd_pack_any, dim3((unsigned)(grid_cap(((S >> 3) + 2) * nd, threads))),
                                           dim3(threads), 0, s, k, v, p, rows, pitch, S, nd))
      return launch_rc(lrc, "bhtd_pack_any");
    return check_launch("bhtd_pack_any");
  }
  if (const cudaError_t lrc = launch_pdl(bhtd_pack_kernel, dim3((unsigned)(grid_cap(((S + 7) >> 3) * nd, threads))),
                                         dim3(threads), 0, s, k, v, p, rows, pitch, S, nd, vec))
    return launch_rc(lrc, "bhtd_pack_kernel");
  return check_launch("bhtd_pack_kernel");
}

int bhtd_unpack(const uint16_t* rows, int64_t pitch, int nd, int64_t S, uint16_t* k, uint16_t* v, int64_t B,
                int64_t H, int64_t T, int64_t D, cudaStream_t s) {
  GSEC_REQUIRE(k && v && rows && B >= 1 && H >= 1 && T >= 1 && D >= 1 && nd >= 1, "bhtd_unpack: bad args");
  Perm p = make_perm(B, H, T, D, 1);
  GSEC_REQUIRE(S * nd >= 2 * p.Tn && pitch >= S, "bhtd_unpack: rows too small");
  const bool vec = (D % 8 == 0) && (S % 8 == 0) && (pitch % 8 == 0) && aligned16(k) && aligned16(v) && aligned16(rows);
  const int threads = 256;
  if (!vec) {
    if (const cudaError_t lrc = launch_pdl(bhtd_unpack_any,
                                           dim3((unsigned)(grid_cap(2 * ((p.Tn >> 3) + 2), threads))), dim3(threads),
                                           0, s, rows, pitch, S, p, k, v))
      return launch_rc(lrc, "bhtd_unpack_any");
    return check_launch("bhtd_unpack_any");
  }
  if (const cudaError_t lrc = launch_pdl(bhtd_unpack_kernel,
                                         dim3((unsigned)(grid_cap((2 * p.Tn + 7) >> 3, threads))), dim3(threads), 0,
                                         s, rows, pitch, S, p, k, v, vec))
    return launch_rc(lrc, "bhtd_unpack_kernel");
  return check_launch("bhtd_unpack_kernel");
}

// ------------------------------------------------- pool rows by slot index --
// The KV pool of an attention backend is [slots, planes, ...] per layer (for
// SGLang's FlashInfer pool: planes K and V). One extend call's delta KV is the
// rows of its slot list; the reference copies them out with two fancy-index
// gathers, after a device-to-host read of the active count
// (bench_ghostserve_rdp.py:449-458). slots_gather writes, for every pool q (a
// layer) and plane p, the rows of the slot list in list order to the byte
// stream position ((q * nplanes + p) * n + i) * row_bytes of a two-segment
// destination (lo[0..split) ++ hi[...]), one launch for every layer of a
// chunk; a slot < 0 gives a zero row, so no count is needed on the host.
// slots_scatter writes such a stream back into the pools (rows of slots < 0
// are skipped). A slot >= pool_rows is an error: the row is zeroed (gather) or
// skipped (scatter) and bit 0 of the layout status is set.
static __device__ unsigned g_layout_status;

namespace {
constexpr int kMaxPools = 128;
struct SlotArgs {
  char* pool[kMaxPools];
  int npools;
  int nplanes;
  int64_t pitch, plane, row_bytes, n, pool_rows, split;
  char* lo;
  char* hi;
};

__device__ __forceinline__ char* seg_at(const SlotArgs& a, int64_t o) {
  return o < a.split ? a.lo + o : a.hi + (o - a.split);
}

template <typename I, bool GATHER>
__global__ void slots_vec(const SlotArgs a, const I* slots) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t vpr = a.row_bytes >> 4;
  const int64_t rows = a.n * a.nplanes * a.npools;
  const int64_t total = vpr * rows;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / vpr;  // (pool * nplanes + plane) * n + list position
    const int64_t x = (v - r * vpr) << 4;
    const int64_t qp = r / a.n, i = r - qp * a.n;
    const int64_t q = qp / a.nplanes, p = qp - q * a.nplanes;
    const int64_t slot = (int64_t)slots[i];
    char* stream = seg_at(a, r * a.row_bytes + x);
    if (slot >= a.pool_rows) {
      if (x == 0) atomicOr(&g_layout_status, 1u);
      if (GATHER) stv(stream, vzero());
    } else if (slot >= 0) {
      char* row = a.pool[q] + slot * a.pitch + p * a.plane + x;
      if (GATHER)
        stv(stream, ldv(row));
      else
        stv(row, ldv(stream));
    } else if (GATHER) {
      stv(stream, vzero());
    }
  }
}
}  // namespace

// --------------------------------------------------- gather of n buffers --
// dst = src[0][0..bytes[0]) ++ src[1][0..bytes[1]) ++ ... moved by bulk copies:
// each CTA's one active thread pulls 16 KiB chunks of the sources into a ring
// of shared-memory stages (cp.async.bulk, no multicast) and pushes each back
// out with a bulk store, four chunks in flight per CTA. The sources may be
// mapped peer buffers, so this is also the plain peer-read copy that bench.py
// times as the NVLink ceiling of a shard placement: the same copy engine the
// encode kernels' producer warps use, with no arithmetic behind it.
static __device__ unsigned g_gather_status;

namespace {
constexpr int kGatherMax = 32;
constexpr int kGChunk = 16384;
constexpr int kGStages = 4;
struct GatherArgs {
  const char* src[kGatherMax];
  int64_t bytes[kGatherMax];
  int64_t dst_off[kGatherMax];   // byte offset of source i in dst
  int64_t items;                 // (largest source's chunk count) x n
  int n;
  char* dst;
};

// Items interleave the sources (item it = chunk it / n of source it % n), so
// the CTAs read every source at once, as the encode kernels read every shard
// of a stripe at once: with peers as sources, all peer links carry traffic
// together. An item past its source's end is empty (len = 0).
__device__ __forceinline__ void gather_item(const GatherArgs& a, int64_t it, const char*& src, char*& dst,
                                            uint32_t& len) {
  const int i = (int)(it % a.n);
  const int64_t off = (it / a.n) * kGChunk;
  const int64_t rest = a.bytes[i] - off;
  len = (uint32_t)(rest <= 0 ? 0 : (rest < kGChunk ? rest : kGChunk));
  src = a.src[i] + off;
  dst = a.dst + a.dst_off[i] + off;
}

// Load one chunk into a stage; an empty chunk completes the stage's phase
// with a plain arrival, so the ring's phase order stays the same.
__device__ __forceinline__ void issue_chunk(unsigned char* stage, const char* src, uint32_t len, uint64_t* bar) {
  if (len == 0) {
    pipe::bar_arrive(bar);
    return;
  }
  pipe::bar_expect_tx(bar, len);
  pipe::bulk_load(stage, src, len, bar);
}

__global__ void __launch_bounds__(32) gather_bulk(const GatherArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGStages * kGChunk);
  if (threadIdx.x == 0) {
    for (int st = 0; st < kGStages; ++st) pipe::bar_init(full + st, 1);
    pipe::bar_init_fence();
  }
  __syncwarp();
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x != 0) return;
  const int64_t items = a.items;
  const char* src;
  char* dst;
  uint32_t len;
  // prologue: the first kGStages chunks of this CTA in flight
  int64_t it = blockIdx.x;
  int64_t issued = 0;  // this CTA's chunks whose loads have been issued, in order
  for (int st = 0; st < kGStages && it + (int64_t)st * gridDim.x < items; ++st) {
    gather_item(a, it + (int64_t)st * gridDim.x, src, dst, len);
    issue_chunk(smem + st * kGChunk, src, len, full + st);
    ++issued;
  }
  for (int64_t k = 0; it < items; ++k, it += gridDim.x) {
    const int st = (int)(k % kGStages);
    if (!pipe::bar_wait(full + st, (uint32_t)((k / kGStages) & 1))) {
      atomicOr(&g_gather_status, 1u);
      // let the loads still in flight land (bounded) before the CTA's shared memory goes away
      for (int64_t q = k + 1; q < issued; ++q)
        (void)pipe::bar_wait(full + q % kGStages, (uint32_t)((q / kGStages) & 1));
      break;
    }
    gather_item(a, it, src, dst, len);
    if (len > 0) {
      pipe::bulk_store(dst, smem + st * kGChunk, len);
      pipe::bulk_commit();
    }
    const int64_t next = it + (int64_t)kGStages * gridDim.x;
    if (next < items) {
      pipe::bulk_wait_read_all();  // the stage's store has read it: refill
      gather_item(a, next, src, dst, len);
      issue_chunk(smem + st * kGChunk, src, len, full + st);
      ++issued;
    }
  }
  pipe::bulk_wait_all();
}
}  // namespace

int copy_gather(const void* const* src, const int64_t* bytes, int n, void* dst, cudaStream_t s) {
  if (n < 1 || n > kGatherMax) {
    set_error("gather: 1..%d sources", kGatherMax);
    return GSEC_EINVAL;
  }
  GatherArgs a{};
  a.n = n;
  a.dst = static_cast<char*>(dst);
  int64_t chunks = 0, off = 0;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] < 0 || (bytes[i] & 15) || (bytes[i] && (!src[i] || !aligned16(src[i])))) {
      set_error("gather: source %d must be 16-byte aligned with a size that is a multiple of 16", i);
      return GSEC_EINVAL;
    }
    a.src[i] = static_cast<const char*>(src[i]);
    a.bytes[i] = bytes[i];
    a.dst_off[i] = off;
    off += bytes[i];
    const int64_t c = (bytes[i] + kGChunk - 1) / kGChunk;
    chunks = c > chunks ? c : chunks;
  }
  const int64_t items = chunks * n;
  a.items = items;
  if (items == 0) return GSEC_OK;
  if (!dst || !aligned16(dst)) {
    set_error("gather: destination must be 16-byte aligned");
    return GSEC_EINVAL;
  }
  const size_t smem = (size_t)kGStages * kGChunk + kGStages * sizeof(uint64_t);
  LaunchCache& cache = launch_cache();
  const int per_sm = cache.blocks_per_sm(gather_bulk, 32, smem);
  if (per_sm < 0) return check_launch("gather_bulk launch shape");
  const int64_t grid = balanced_grid(items, (int64_t)sm_count() * per_sm);
  return launch_rc(launch_pdl(gather_bulk, dim3((unsigned)grid), dim3(32), smem, s, a), "gather_bulk");
}

unsigned gather_device_status(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gather_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_gather_status, &z, sizeof(z));
  }
  return v;
}

unsigned layout_device_status(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_layout_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_layout_status, &z, sizeof(z));
  }
  return v;
}

int slots_move(bool gather, void* const* pools, int npools, int64_t pitch, int64_t plane, int nplanes,
               int64_t row_bytes, const void* slots, int slot_bytes, int64_t n, int64_t pool_rows, void* lo,
               void* hi, int64_t split, cudaStream_t s) {
  if (n == 0) return GSEC_OK;
  if (npools < 1 || npools > kMaxPools) {
    set_error("slot rows: 1..%d pools", kMaxPools);
    return GSEC_EINVAL;
  }
  const int64_t total = (int64_t)npools * nplanes * n * row_bytes;
  const bool two = hi != nullptr && split < total;
  if (!aligned16(lo) || (two && (!aligned16(hi) || (split & 15) || split < 0)) || (pitch & 15) || (plane & 15) ||
      (row_bytes & 15) || row_bytes <= 0) {
    set_error("slot rows: pools, buffer, split, pitch, plane offset and row bytes must be 16-byte aligned");
    return GSEC_EINVAL;
  }
  SlotArgs a{};
  for (int q = 0; q < npools; ++q) {
    if (!pools[q] || !aligned16(pools[q])) {
      set_error("slot rows: pool %d is null or not 16-byte aligned", q);
      return GSEC_EINVAL;
    }
    a.pool[q] = static_cast<char*>(pools[q]);
  }
  a.npools = npools;
  a.nplanes = nplanes;
  a.pitch = pitch;
  a.plane = plane;
  a.row_bytes = row_bytes;
  a.n = n;
  a.pool_rows = pool_rows;
  a.lo = static_cast<char*>(lo);
  a.hi = two ? static_cast<char*>(hi) : a.lo;
  a.split = two ? split : INT64_MAX;
  const int threads = 256;
  const dim3 grid((unsigned)grid_cap((row_bytes >> 4) * n * nplanes * npools, threads));
  cudaError_t rc;
  if (gather)
    rc = slot_bytes == 8 ? launch_pdl(slots_vec<int64_t, true>, grid, dim3(threads), 0, s, a,
                                      static_cast<const int64_t*>(slots))
                         : launch_pdl(slots_vec<int32_t, true>, grid, dim3(threads), 0, s, a,
                                      static_cast<const int32_t*>(slots));
  else
    rc = slot_bytes == 8 ? launch_pdl(slots_vec<int64_t, false>, grid, dim3(threads), 0, s, a,
                                      static_cast<const int64_t*>(slots))
                         : launch_pdl(slots_vec<int32_t, false>, grid, dim3(threads), 0, s, a,
                                      static_cast<const int32_t*>(slots));
  return launch_rc(rc, gather ? "slots_gather" : "slots_scatter");
}

}  // namespace gsec
