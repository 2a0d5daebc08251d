/*
 * oracle.c — C/OpenMP restatement of the KV erasure codes, used as the timed
 * CPU baseline and as a second, independent CPU check.  TEST INFRASTRUCTURE:
 * never linked into or called by the product.
 *
 * The reference has no CPU encoder (all its encoders are CUDA kernels), so
 * this is a port of the same arithmetic to host cores:
 *   orc_xor_encode      benchmark/xor/kernel.cu:32-40 (parity half of encode_xor_kernel)
 *   orc_rdpref_parity   benchmark/rdp/kernel.cu:76-107 and bench_ghostserve_rdp.py:121-150
 *   orc_rs16_encode     benchmark/rs/kernel.cu:67-102 with the tables of benchmark/rs/main.py:39-54
 *   orc_rdp_encode      textbook RDP (Corbett et al., FAST 2004), no reference code
 *   orc_rs8_encode      RS over GF(2^8)/0x11d, Cauchy generator, no reference code
 * Work is split over OpenMP threads by position (or stripe); XOR runs on
 * 64-bit words.
 */
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define API __attribute__((visibility("default")))

static void set_threads(int threads) {
  if (threads > 0) omp_set_num_threads(threads);
}

API int orc_max_threads(void) { return omp_get_max_threads(); }

/* ------------------------------------------------------------------ XOR --- */
API void orc_xor_encode(const uint8_t* const* data, int k, int64_t n, uint8_t* parity, int threads) {
  set_threads(threads);
  const int64_t nw = n / 8;
#pragma omp parallel for schedule(static)
  for (int64_t w = 0; w < nw; ++w) {
    uint64_t acc = 0;
    for (int i = 0; i < k; ++i) {
      uint64_t x;
      memcpy(&x, data[i] + 8 * w, 8);
      acc ^= x;
    }
    memcpy(parity + 8 * w, &acc, 8);
  }
  for (int64_t b = nw * 8; b < n; ++b) {
    uint8_t acc = 0;
    for (int i = 0; i < k; ++i) acc ^= data[i][b];
    parity[b] = acc;
  }
}

/* ------------------------------------------------------------ textbook RDP */
/* Stripe t of every shard: (p-1) units of `unit` bytes; cell (r, c) on
 * diagonal (r + c) mod p; columns k..p-2 are zero; diagonal p-1 not stored.
 * data shards hold data_bytes bytes (zero past the end); P and Q hold whole
 * stripes. */
API void orc_rdp_encode(const uint8_t* const* data, int k, int p, int64_t unit, int64_t data_bytes,
                        uint8_t* P, uint8_t* Q, int threads) {
  set_threads(threads);
  const int64_t sb = (int64_t)(p - 1) * unit;
  const int64_t ns = (data_bytes + sb - 1) / sb;
  const int64_t nw = unit / 8;
#pragma omp parallel
  {
    uint64_t* q = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)p * (size_t)nw);
    uint64_t* prow = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nw);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < ns; ++t) {
      memset(q, 0, sizeof(uint64_t) * (size_t)p * (size_t)nw);
      for (int r = 0; r < p - 1; ++r) {
        const int64_t off = t * sb + (int64_t)r * unit;
        memset(prow, 0, sizeof(uint64_t) * (size_t)nw);
        for (int c = 0; c < k; ++c) {
          uint64_t* qd = q + (size_t)((r + c) % p) * (size_t)nw;
          if (off + unit <= data_bytes) {
            const uint64_t* src = (const uint64_t*)(data[c] + off);
            for (int64_t w = 0; w < nw; ++w) {
              prow[w] ^= src[w];
              qd[w] ^= src[w];
            }
          } else if (off < data_bytes) {
            uint64_t tmp[512];
            for (int64_t w0 = 0; w0 < nw; w0 += 512) {
              const int64_t cnt = nw - w0 < 512 ? nw - w0 : 512;
              memset(tmp, 0, sizeof(tmp));
              int64_t avail = data_bytes - off - w0 * 8;
              if (avail > cnt * 8) avail = cnt * 8;
              if (avail > 0) memcpy(tmp, data[c] + off + w0 * 8, (size_t)avail);
              for (int64_t w = 0; w < cnt; ++w) {
                prow[w0 + w] ^= tmp[w];
                qd[w0 + w] ^= tmp[w];
              }
            }
          }
        }
        memcpy(P + off, prow, (size_t)unit);
        uint64_t* qd = q + (size_t)((r + p - 1) % p) * (size_t)nw;
        for (int64_t w = 0; w < nw; ++w) qd[w] ^= prow[w];
      }
      for (int d = 0; d < p - 1; ++d) memcpy(Q + t * sb + (int64_t)d * unit, q + (size_t)d * (size_t)nw, (size_t)unit);
    }
    free(q);
    free(prow);
  }
}

/* ------------------------------------------------------------------ GF --- */
static uint32_t gf8_mul(uint32_t a, uint32_t b) {
  uint32_t r = 0;
  for (int i = 0; i < 8; ++i) {
    if (b & 1u) r ^= a;
    b >>= 1;
    a <<= 1;
    if (a & 0x100u) a ^= 0x11du;
  }
  return r & 0xffu;
}

static uint32_t gf8_inv(uint32_t a) {
  for (uint32_t x = 1; x < 256; ++x)
    if (gf8_mul(a, x) == 1) return x;
  return 0;
}

/* Cauchy parity: C[j][i] = 1 / ((k + j) ^ i). One 256-entry product table per
 * coefficient. */
API void orc_rs8_encode(const uint8_t* const* data, int k, int m, int64_t n, uint8_t* const* parity, int threads) {
  set_threads(threads);
  uint8_t* tab = (uint8_t*)malloc((size_t)m * (size_t)k * 256);
  for (int j = 0; j < m; ++j)
    for (int i = 0; i < k; ++i) {
      const uint32_t c = gf8_inv((uint32_t)((k + j) ^ i));
      for (int x = 0; x < 256; ++x) tab[((size_t)j * k + i) * 256 + x] = (uint8_t)gf8_mul(c, (uint32_t)x);
    }
  const int64_t blk = 4096;
  const int64_t nb = (n + blk - 1) / blk;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t lo = b * blk, hi = lo + blk < n ? lo + blk : n;
    for (int j = 0; j < m; ++j) {
      uint8_t* out = parity[j];
      memset(out + lo, 0, (size_t)(hi - lo));
      for (int i = 0; i < k; ++i) {
        const uint8_t* t = tab + ((size_t)j * k + i) * 256;
        const uint8_t* src = data[i];
        for (int64_t x = lo; x < hi; ++x) out[x] ^= t[src[x]];
      }
    }
  }
  free(tab);
}

/* benchmark/rs/main.py:39-54 tables, then benchmark/rs/kernel.cu:84-101. */
API void orc_rs16_encode(const uint16_t* data_padded, int k, int m, int64_t s, uint16_t* parity_rows,
                         int threads) {
  set_threads(threads);
  uint16_t* gexp = (uint16_t*)malloc(sizeof(uint16_t) * 2 * 65535);
  uint16_t* glog = (uint16_t*)calloc(65536, sizeof(uint16_t));
  uint32_t x = 1;
  for (int i = 0; i < 65535; ++i) {
    gexp[i] = (uint16_t)x;
    glog[x] = (uint16_t)i;
    x <<= 1;
    if (x & 0x10000u) x ^= 0x1100bu;
  }
  for (int i = 65535; i < 2 * 65535; ++i) gexp[i] = gexp[i - 65535];
#pragma omp parallel for schedule(static)
  for (int64_t pos = 0; pos < s; ++pos) {
    for (int p = 0; p < m; ++p) {
      uint16_t acc = 0;
      const int base = p + 1;
      for (int kk = 0; kk < k; ++kk) {
        const uint16_t v = data_padded[(int64_t)kk * s + pos];
        if (v) {
          const uint16_t coef = gexp[(base * kk) % 65535];
          int e = (int)glog[v] + (int)glog[coef];
          if (e >= 65535) e -= 65535;
          acc ^= gexp[e];
        }
      }
      parity_rows[(int64_t)p * s + pos] = acc;
    }
  }
  free(gexp);
  free(glog);
}

/* -------------------------------------------------------------- RDP-ref --- */
API void orc_rdpref_parity(uint16_t* rows, int nd, int64_t S, int star_base, int threads) {
  set_threads(threads);
  uint16_t* P = rows + (int64_t)nd * S;
  uint16_t* Q = rows + (int64_t)(nd + 1) * S;
#pragma omp parallel for schedule(static)
  for (int64_t d = 0; d < S; ++d) {
    uint16_t pa = 0, qa = 0;
    for (int r = 0; r < nd; ++r) {
      pa ^= rows[(int64_t)r * S + d];
      int64_t c = (d - r) % S;
      if (c < 0) c += S;
      const int star = (int)(((long long)star_base + r) % S);
      if (c == star) continue;
      qa ^= rows[(int64_t)r * S + c];
    }
    P[d] = pa;
    Q[d] = qa;
  }
}
