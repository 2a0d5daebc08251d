// api.cu — the extern "C" entry points of libgsec (declared in include/gsec.h):
// argument checks, host-side code math (GF inverses, decode matrices, RDP
// masks), kernel dispatch and CUDA IPC peer mapping.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "layout.cuh"
#include "linear.cuh"
#include "rdp.cuh"
#include "rdpref.cuh"

namespace gsec {

// ---------------------------------------------------------------- errors ----
static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
}
const char* last_error() { return g_err.c_str(); }

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return GSEC_ECUDA;
  }
  return GSEC_OK;
}

int launch_rc(cudaError_t rc, const char* what) {
  if (rc == cudaSuccess) return check_launch(what);
  cudaGetLastError();
  set_error("%s: %s", what, cudaGetErrorString(rc));
  return GSEC_ECUDA;
}

int current_device() {
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess ? dev : -1;
}

LaunchCache& launch_cache() {
  static LaunchCache cache;
  return cache;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// -------------------------------------------------------------- GF tables ---
namespace {
struct Gf8Tables {
  uint8_t exp[512];
  uint8_t log[256];
  Gf8Tables() {
    uint32_t x = 1;
    for (int i = 0; i < 255; ++i) {
      exp[i] = (uint8_t)x;
      log[x] = (uint8_t)i;
      x <<= 1;
      if (x & 0x100u) x ^= 0x11du;
    }
    for (int i = 255; i < 512; ++i) exp[i] = exp[i - 255];
    log[0] = 0;
  }
};
const Gf8Tables& gf8t() {
  static const Gf8Tables t;
  return t;
}

// The reference's GF(2^16) tables (benchmark/rs/main.py:39-54): exp has 2*65535
// entries (second half repeats the first), log[0] stays 0.
struct Gf16Tables {
  std::vector<uint16_t> exp, log;
  Gf16Tables() : exp(2 * 65535), log(65536, 0) {
    uint32_t x = 1;
    for (int i = 0; i < 65535; ++i) {
      exp[i] = (uint16_t)x;
      log[x] = (uint16_t)i;
      x <<= 1;
      if (x & 0x10000u) x ^= 0x1100bu;
    }
    for (int i = 65535; i < 2 * 65535; ++i) exp[i] = exp[i - 65535];
  }
};
const Gf16Tables& gf16t() {
  static const Gf16Tables t;
  return t;
}
}  // namespace

uint8_t gf8_inv(uint8_t a) {
  const Gf8Tables& t = gf8t();
  return a == 0 ? 0 : t.exp[(255 - t.log[a]) % 255];
}
static uint8_t gf8_mul_h(uint8_t a, uint8_t b) {
  const Gf8Tables& t = gf8t();
  return (a == 0 || b == 0) ? 0 : t.exp[t.log[a] + t.log[b]];
}
uint16_t gf16_exp(int e) { return gf16t().exp[e]; }
uint16_t gf16_log(uint16_t a) { return gf16t().log[a]; }
// gf_mul / gf_div exactly as benchmark/rs/kernel.cu:16-33.
uint16_t gf16_mul_tab(uint16_t a, uint16_t b) {
  if (a == 0 || b == 0) return 0;
  int s = (int)gf16t().log[a] + (int)gf16t().log[b];
  if (s >= 65535) s -= 65535;
  return gf16t().exp[s];
}
uint16_t gf16_div_tab(uint16_t a, uint16_t b) {
  if (a == 0 || b == 0) return 0;
  int d = (int)gf16t().log[a] - (int)gf16t().log[b];
  if (d < 0) d += 65535;
  return gf16t().exp[d];
}

// ----------------------------------------------------------- code helpers ---
namespace {

// RS8 generator: rows 0..k-1 identity, parity row j = k + j has entries
// C[j][i] = 1 / (x_j + y_i) with x_j = k + j, y_i = i (addition is XOR), no
// normalisation.  x and y sets are disjoint and distinct, so every square
// submatrix of C is invertible and the code is MDS for k + m <= 256.
uint8_t rs8_gen(int k, int row, int col) {
  if (row < k) return row == col ? 1 : 0;
  return gf8_inv((uint8_t)(row ^ col));
}

// Invert an n x n matrix over GF(2^8); returns false if singular.
bool gf8_invert(std::vector<uint8_t>& a, int n, std::vector<uint8_t>& inv) {
  inv.assign((size_t)n * n, 0);
  for (int i = 0; i < n; ++i) inv[(size_t)i * n + i] = 1;
  for (int c = 0; c < n; ++c) {
    int piv = -1;
    for (int r = c; r < n; ++r)
      if (a[(size_t)r * n + c]) { piv = r; break; }
    if (piv < 0) return false;
    if (piv != c)
      for (int j = 0; j < n; ++j) {
        std::swap(a[(size_t)piv * n + j], a[(size_t)c * n + j]);
        std::swap(inv[(size_t)piv * n + j], inv[(size_t)c * n + j]);
      }
    const uint8_t s = gf8_inv(a[(size_t)c * n + c]);
    for (int j = 0; j < n; ++j) {
      a[(size_t)c * n + j] = gf8_mul_h(a[(size_t)c * n + j], s);
      inv[(size_t)c * n + j] = gf8_mul_h(inv[(size_t)c * n + j], s);
    }
    for (int r = 0; r < n; ++r) {
      if (r == c || a[(size_t)r * n + c] == 0) continue;
      const uint8_t f = a[(size_t)r * n + c];
      for (int j = 0; j < n; ++j) {
        a[(size_t)r * n + j] ^= gf8_mul_h(f, a[(size_t)c * n + j]);
        inv[(size_t)r * n + j] ^= gf8_mul_h(f, inv[(size_t)c * n + j]);
      }
    }
  }
  return true;
}

int check_code(const gsec_code* code) {
  GSEC_REQUIRE(code != nullptr, "code is null");
  switch (code->scheme) {
    case GSEC_SCHEME_XOR:
      GSEC_REQUIRE(code->k >= 1 && code->k <= kLinMaxIn - 1, "XOR: k=%d must be in [1, %d]", code->k, kLinMaxIn - 1);
      GSEC_REQUIRE(code->m == 1, "XOR: m=%d must be 1", code->m);
      return GSEC_OK;
    case GSEC_SCHEME_RS8:
      GSEC_REQUIRE(code->k >= 1 && code->k <= kLinMaxIn, "RS8: k=%d must be in [1, %d]", code->k, kLinMaxIn);
      GSEC_REQUIRE(code->m >= 1 && code->m <= kLinMaxOut, "RS8: m=%d must be in [1, %d]", code->m, kLinMaxOut);
      return GSEC_OK;
    case GSEC_SCHEME_RDP:
      if (!rdp_prime_supported(code->p)) {
        set_error("RDP: p=%d not supported (3,5,7,11,13,17)", code->p);
        return GSEC_EUNSUPPORTED;
      }
      GSEC_REQUIRE(code->k >= 1 && code->k <= code->p - 1, "RDP: k=%d must be in [1, p-1=%d]", code->k, code->p - 1);
      GSEC_REQUIRE(code->m == 2, "RDP: m=%d must be 2", code->m);
      GSEC_REQUIRE(code->unit >= 16 && code->unit % 16 == 0, "RDP: unit=%lld must be a positive multiple of 16",
                   (long long)code->unit);
      return GSEC_OK;
    default:
      set_error("unknown scheme %d", code->scheme);
      return GSEC_EINVAL;
  }
}

int64_t parity_len(const gsec_code* c, int64_t data_bytes) {
  if (c->scheme == GSEC_SCHEME_RDP) {
    const int64_t sb = (int64_t)(c->p - 1) * c->unit;
    return (data_bytes + sb - 1) / sb * sb;
  }
  return data_bytes;
}

// Range granule: RDP works on whole stripes, the others on 16-byte vectors.
int64_t granule(const gsec_code* c) {
  return c->scheme == GSEC_SCHEME_RDP ? (int64_t)(c->p - 1) * c->unit : 16;
}

int check_range(const gsec_code* c, int64_t data_bytes, int64_t begin, int64_t end) {
  GSEC_REQUIRE(data_bytes > 0 && data_bytes % 16 == 0, "data_bytes=%lld must be a positive multiple of 16",
               (long long)data_bytes);
  const int64_t plen = parity_len(c, data_bytes);
  const int64_t g = granule(c);
  GSEC_REQUIRE(begin >= 0 && begin <= end && end <= plen, "range [%lld, %lld) outside [0, %lld)",
               (long long)begin, (long long)end, (long long)plen);
  GSEC_REQUIRE(begin % g == 0 && (end % g == 0 || end == plen), "range [%lld, %lld) not aligned to %lld bytes",
               (long long)begin, (long long)end, (long long)g);
  return GSEC_OK;
}

}  // namespace
}  // namespace gsec

using namespace gsec;

// ===================================================================== C ABI ==
extern "C" {

const char* gsec_last_error(void) { return last_error(); }
const char* gsec_version(void) { return "gsec 0.1.0 (sm_100a)"; }

int gsec_device_status(uint32_t* status, int32_t clear) {
  GSEC_REQUIRE(status != nullptr, "status is null");
  if (cudaDeviceSynchronize() != cudaSuccess) return check_launch("device synchronize");
  const unsigned v1 = rdp_device_status(clear != 0);
  const unsigned v2 = linear_device_status(clear != 0);
  const unsigned v3 = layout_device_status(clear != 0);
  const unsigned v4 = gather_device_status(clear != 0);
  const unsigned v = (v1 == 0xffffffffu || v2 == 0xffffffffu || v3 == 0xffffffffu || v4 == 0xffffffffu)
                         ? 0xffffffffu
                         : (v1 | (v2 << 8) | (v3 << 16) | (v4 << 24));
  if (v == 0xffffffffu) {
    set_error("cannot read the device status word");
    return GSEC_ECUDA;
  }
  *status = v;
  return GSEC_OK;
}

int gsec_parity_bytes(const gsec_code* code, int64_t data_bytes, int64_t* out) {
  int rc = check_code(code);
  if (rc) return rc;
  GSEC_REQUIRE(out != nullptr && data_bytes >= 0, "bad output pointer or size");
  *out = parity_len(code, data_bytes);
  return GSEC_OK;
}

namespace {
// True if any of the pointers lies in another GPU's memory (a peer buffer
// mapped with gsec_ipc_import): such inputs are read by the bulk-copy kernels,
// which keep more bytes in flight over NVLink than 16-byte loads do.
bool any_remote(const void* const* p, int n) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  for (int i = 0; i < n; ++i) {
    if (p[i] == nullptr) continue;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p[i]) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (attr.type == cudaMemoryTypeDevice && attr.device != dev) return true;
  }
  return false;
}
}  // namespace

int gsec_encode(const gsec_code* code, const void* const* data_lo, const void* const* data_hi, int64_t split,
                int64_t data_bytes, void* const* parity, int64_t begin, int64_t end, gsec_stream_t stream) {
  int rc = check_code(code);
  if (rc) return rc;
  rc = check_range(code, data_bytes, begin, end);
  if (rc) return rc;
  GSEC_REQUIRE(data_lo != nullptr && parity != nullptr, "null shard array");
  const bool two_seg = data_hi != nullptr && split < data_bytes;
  if (two_seg) GSEC_REQUIRE(split >= 0 && split % 16 == 0, "split=%lld must be a multiple of 16", (long long)split);
  const int64_t sp = two_seg ? split : INT64_MAX;
  const int k = code->k, m = code->m;
  for (int i = 0; i < k; ++i) {
    GSEC_REQUIRE(data_lo[i] && aligned16(data_lo[i]), "data shard %d pointer null or not 16-byte aligned", i);
    if (two_seg) GSEC_REQUIRE(data_hi[i] && aligned16(data_hi[i]), "data shard %d high segment bad", i);
  }
  for (int j = 0; j < m; ++j)
    GSEC_REQUIRE(parity[j] && aligned16(parity[j]), "parity shard %d pointer null or not 16-byte aligned", j);
  if (end == begin) return GSEC_OK;
  const cudaStream_t s = as_stream(stream);

  if (code->scheme == GSEC_SCHEME_RDP) {
    RdpEncodeArgs a{};
    for (int i = 0; i < k; ++i) {
      a.d_lo[i] = static_cast<const char*>(data_lo[i]);
      a.d_hi[i] = two_seg ? static_cast<const char*>(data_hi[i]) : a.d_lo[i];
    }
    a.parity[0] = static_cast<char*>(parity[0]);
    a.parity[1] = static_cast<char*>(parity[1]);
    a.split = sp;
    a.data_bytes = data_bytes;
    a.unit = code->unit;
    const int64_t sb = (int64_t)(code->p - 1) * code->unit;
    a.s_begin = begin / sb;
    a.s_end = (end + sb - 1) / sb;
    a.k = k;
    a.p = code->p;
    if (code->p <= 3) a.remote = any_remote(data_lo, k) || (two_seg && any_remote(data_hi, k));
    return rdp_encode(a, s);
  }

  LinearPass a{};
  a.nin = k;
  a.nout = m;
  a.split = sp;
  a.begin = begin;
  a.end = end;
  a.field = code->scheme == GSEC_SCHEME_XOR ? Field::XOR : Field::GF8;
  for (int i = 0; i < k; ++i) {
    a.in_lo[i] = static_cast<const char*>(data_lo[i]);
    a.in_hi[i] = two_seg ? static_cast<const char*>(data_hi[i]) : a.in_lo[i];
  }
  for (int j = 0; j < m; ++j) {
    a.out_lo[j] = static_cast<char*>(parity[j]);
    a.out_hi[j] = two_seg ? a.out_lo[j] + sp : a.out_lo[j];
    a.out_end[j] = end;
    for (int i = 0; i < k; ++i) a.coef[j][i] = rs8_gen(k, k + j, i);
  }
  if (a.field == Field::XOR && k <= 3) a.remote = any_remote(data_lo, k) || (two_seg && any_remote(data_hi, k));
  return run_linear(a, s);
}

int gsec_decode(const gsec_code* code, void* const* shard_lo, void* const* shard_hi, int64_t split,
                int64_t data_bytes, const int32_t* erased, int32_t nerased, int64_t begin, int64_t end,
                gsec_stream_t stream) {
  int rc = check_code(code);
  if (rc) return rc;
  rc = check_range(code, data_bytes, begin, end);
  if (rc) return rc;
  const int k = code->k, m = code->m, n = k + m;
  GSEC_REQUIRE(shard_lo != nullptr, "null shard array");
  GSEC_REQUIRE(nerased >= 0 && (nerased == 0 || erased != nullptr), "bad erased list");
  if (nerased > m) {
    set_error("%d erasures exceed the %d parity shards", nerased, m);
    return GSEC_EUNRECOVERABLE;
  }
  std::vector<bool> is_erased(n, false);
  for (int e = 0; e < nerased; ++e) {
    GSEC_REQUIRE(erased[e] >= 0 && erased[e] < n, "erased index %d out of [0, %d)", erased[e], n);
    GSEC_REQUIRE(!is_erased[erased[e]], "erased index %d repeated", erased[e]);
    is_erased[erased[e]] = true;
  }
  if (nerased == 0 || end == begin) return GSEC_OK;
  const bool two_seg = shard_hi != nullptr && split < data_bytes;
  if (two_seg) GSEC_REQUIRE(split >= 0 && split % 16 == 0, "split=%lld must be a multiple of 16", (long long)split);
  const int64_t sp = two_seg ? split : INT64_MAX;
  for (int i = 0; i < n; ++i) {
    GSEC_REQUIRE(shard_lo[i] && aligned16(shard_lo[i]), "shard %d pointer null or not 16-byte aligned", i);
    if (two_seg && i < k) GSEC_REQUIRE(shard_hi[i] && aligned16(shard_hi[i]), "shard %d high segment bad", i);
  }
  auto lo = [&](int i) { return static_cast<char*>(shard_lo[i]); };
  auto hi = [&](int i) -> char* {
    if (!two_seg) return lo(i);
    return i < k ? static_cast<char*>(shard_hi[i]) : lo(i) + sp;
  };
  const cudaStream_t s = as_stream(stream);

  if (code->scheme == GSEC_SCHEME_RDP) {
    const int p = code->p;
    RdpDecodeArgs a{};
    a.p = p;
    a.split = sp;
    a.data_bytes = data_bytes;
    a.unit = code->unit;
    const int64_t sb = (int64_t)(p - 1) * code->unit;
    a.s_begin = begin / sb;
    a.s_end = (end + sb - 1) / sb;
    auto col_of = [&](int i) { return i < k ? i : (i == k ? p - 1 : p); };
    int cols[2];
    for (int e = 0; e < nerased; ++e) cols[e] = col_of(erased[e]);
    rc = rdp_solve_masks(p, cols, nerased, a.mask);
    if (rc) return rc;
    a.alive = 0;
    for (int i = 0; i < n; ++i) {
      const int c = col_of(i);
      a.lo[c] = lo(i);
      a.hi[c] = hi(i);
      if (!is_erased[i]) a.alive |= 1u << c;
    }
    a.nout = nerased;
    for (int e = 0; e < nerased; ++e) {
      a.out_col[e] = cols[e];
      a.out_lo[e] = lo(erased[e]);
      a.out_hi[e] = hi(erased[e]);
    }
    rdp_build_program(a);
    if (code->p <= 3) {
      std::vector<const void*> in;
      for (int i = 0; i < n; ++i)
        if (!is_erased[i]) {
          in.push_back(lo(i));
          in.push_back(hi(i));
        }
      a.remote = any_remote(in.data(), (int)in.size());
    }
    return rdp_decode(a, s);
  }

  LinearPass a{};
  a.split = sp;
  a.begin = begin;
  a.end = end;
  if (code->scheme == GSEC_SCHEME_XOR) {
    a.field = Field::XOR;
    for (int i = 0; i < n; ++i)
      if (!is_erased[i]) {
        a.in_lo[a.nin] = lo(i);
        a.in_hi[a.nin] = hi(i);
        ++a.nin;
      }
    a.nout = 1;
    a.out_lo[0] = lo(erased[0]);
    a.out_hi[0] = hi(erased[0]);
    a.out_end[0] = erased[0] < k ? data_bytes : end;
    if (a.nin <= 3) {
      std::vector<const void*> in(a.in_lo, a.in_lo + a.nin);
      in.insert(in.end(), a.in_hi, a.in_hi + a.nin);
      a.remote = any_remote(in.data(), (int)in.size());
    }
    return run_linear(a, s);
  }

  // RS8: survivors = first k shards that are not erased; output rows = G[e] * S^-1.
  a.field = Field::GF8;
  std::vector<int> surv;
  for (int i = 0; i < n && (int)surv.size() < k; ++i)
    if (!is_erased[i]) surv.push_back(i);
  std::vector<uint8_t> sm((size_t)k * k), inv;
  for (int r = 0; r < k; ++r)
    for (int c = 0; c < k; ++c) sm[(size_t)r * k + c] = rs8_gen(k, surv[r], c);
  if (!gf8_invert(sm, k, inv)) {
    set_error("RS8 survivor matrix is singular");
    return GSEC_EUNRECOVERABLE;
  }
  a.nin = k;
  for (int r = 0; r < k; ++r) {
    a.in_lo[r] = lo(surv[r]);
    a.in_hi[r] = hi(surv[r]);
  }
  a.nout = nerased;
  for (int e = 0; e < nerased; ++e) {
    const int row = erased[e];
    for (int c = 0; c < k; ++c) {
      uint8_t acc = 0;
      for (int t = 0; t < k; ++t) acc ^= gf8_mul_h(rs8_gen(k, row, t), inv[(size_t)t * k + c]);
      a.coef[e][c] = acc;
    }
    a.out_lo[e] = lo(row);
    a.out_hi[e] = hi(row);
    a.out_end[e] = row < k ? data_bytes : end;
  }
  return run_linear(a, s);
}

// ------------------------------------------------------------------ layout --
int gsec_rows_pack(const void* src0, int64_t len0, const void* src1, int64_t len1, void* rows, int64_t pitch,
                   int64_t row_bytes, int32_t nrows, gsec_stream_t stream) {
  return rows_pack(src0, len0, src1, len1, rows, pitch, row_bytes, nrows, as_stream(stream));
}

int gsec_rows_unpack(const void* rows, int64_t pitch, int64_t row_bytes, int32_t nrows, void* dst0, int64_t len0,
                     void* dst1, int64_t len1, gsec_stream_t stream) {
  return rows_unpack(rows, pitch, row_bytes, nrows, dst0, len0, dst1, len1, as_stream(stream));
}

namespace {
// Every plane of a slot's record must lie inside the record: planes at byte
// offsets 0, plane, ..., (nplanes-1)*plane, each row_bytes long, in pitch bytes.
bool slot_geometry_ok(int64_t pitch, int64_t plane, int32_t nplanes, int64_t row_bytes) {
  if (pitch <= 0 || plane < 0 || row_bytes <= 0 || nplanes < 1) return false;
  if (plane > 0 && (int64_t)(nplanes - 1) > (pitch - row_bytes) / plane) return false;
  return (int64_t)(nplanes - 1) * plane + row_bytes <= pitch;
}
}  // namespace

int gsec_slots_gather(const void* pool, int64_t pitch, int64_t plane, int32_t nplanes, int64_t row_bytes,
                      const void* slots, int32_t slot_bytes, int64_t n, int64_t pool_rows, void* dst,
                      gsec_stream_t stream) {
  void* pools[1] = {const_cast<void*>(pool)};
  return gsec_slots_gather_pools(pools, 1, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows, dst,
                                 nullptr, INT64_MAX, stream);
}

int gsec_slots_scatter(void* pool, int64_t pitch, int64_t plane, int32_t nplanes, int64_t row_bytes,
                       const void* slots, int32_t slot_bytes, int64_t n, int64_t pool_rows, const void* src,
                       gsec_stream_t stream) {
  void* pools[1] = {pool};
  return gsec_slots_scatter_pools(pools, 1, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows,
                                  src, nullptr, INT64_MAX, stream);
}

namespace {
int slots_args_ok(const void* const* pools, int32_t npools, int64_t pitch, int64_t plane, int32_t nplanes,
                  int64_t row_bytes, const void* slots, int32_t slot_bytes, int64_t n, int64_t pool_rows,
                  const void* lo) {
  GSEC_REQUIRE(pools != nullptr && lo != nullptr && (n == 0 || slots != nullptr), "null pointer");
  GSEC_REQUIRE(npools >= 1, "npools=%d must be >= 1", npools);
  for (int q = 0; q < npools; ++q) GSEC_REQUIRE(pools[q] != nullptr, "null pointer (pool %d)", q);
  GSEC_REQUIRE(slot_bytes == 4 || slot_bytes == 8, "slot_bytes=%d must be 4 or 8", slot_bytes);
  GSEC_REQUIRE(nplanes >= 1 && n >= 0 && pool_rows >= 0, "bad nplanes/n/pool_rows");
  GSEC_REQUIRE(slot_geometry_ok(pitch, plane, nplanes, row_bytes),
               "slot record: need pitch > 0, plane >= 0 and (nplanes-1)*plane + row_bytes <= pitch");
  return GSEC_OK;
}
}  // namespace

int gsec_slots_gather_pools(void* const* pools, int32_t npools, int64_t pitch, int64_t plane, int32_t nplanes,
                            int64_t row_bytes, const void* slots, int32_t slot_bytes, int64_t n, int64_t pool_rows,
                            void* dst_lo, void* dst_hi, int64_t split, gsec_stream_t stream) {
  const int rc = slots_args_ok(pools, npools, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows,
                               dst_lo);
  if (rc) return rc;
  return slots_move(true, pools, npools, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows, dst_lo,
                    dst_hi, split, as_stream(stream));
}

int gsec_slots_scatter_pools(void* const* pools, int32_t npools, int64_t pitch, int64_t plane, int32_t nplanes,
                             int64_t row_bytes, const void* slots, int32_t slot_bytes, int64_t n, int64_t pool_rows,
                             const void* src_lo, const void* src_hi, int64_t split, gsec_stream_t stream) {
  const int rc = slots_args_ok(pools, npools, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows,
                               src_lo);
  if (rc) return rc;
  return slots_move(false, pools, npools, pitch, plane, nplanes, row_bytes, slots, slot_bytes, n, pool_rows,
                    const_cast<void*>(src_lo), const_cast<void*>(src_hi), split, as_stream(stream));
}

int gsec_copy_gather(const void* const* src, const int64_t* bytes, int32_t n, void* dst, gsec_stream_t stream) {
  GSEC_REQUIRE(src != nullptr && bytes != nullptr, "null source array");
  return copy_gather(src, bytes, n, dst, as_stream(stream));
}

int gsec_copy_async(void* dst, const void* src, int64_t bytes, gsec_stream_t stream) {
  GSEC_REQUIRE(bytes >= 0, "bytes < 0");
  if (bytes == 0) return GSEC_OK;
  GSEC_REQUIRE(dst != nullptr && src != nullptr, "null pointer");
  if (cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, as_stream(stream)) != cudaSuccess)
    return check_launch("cudaMemcpyAsync");
  return GSEC_OK;
}

// ------------------------------------------------------------- XOR compat ---
namespace {
// Row r of a row-major shard buffer as a contiguous LinearPass input/output.
void set_row_in(LinearPass& a, const char* base, int64_t pitch, int r) {
  a.in_lo[a.nin] = base + (int64_t)r * pitch;
  a.in_hi[a.nin] = a.in_lo[a.nin];
  ++a.nin;
}
void set_row_out(LinearPass& a, char* p, int64_t end) {
  a.out_lo[a.nout] = p;
  a.out_hi[a.nout] = p;
  a.out_end[a.nout] = end;
  ++a.nout;
}
}  // namespace

int gsec_xor_encode(const uint8_t* data_padded, uint8_t* shards, int32_t data_shards, int64_t shard_size,
                    int64_t pitch, gsec_stream_t stream) {
  GSEC_REQUIRE(shards != nullptr, "shards is null");
  GSEC_REQUIRE(data_shards >= 1 && data_shards <= kLinMaxIn, "data_shards=%d must be in [1, %d]", data_shards,
               kLinMaxIn);
  GSEC_REQUIRE(shard_size >= 1 && pitch >= shard_size, "bad shard_size/pitch");
  const cudaStream_t s = as_stream(stream);
  const bool rows_aligned = aligned16(shards) && shard_size % 16 == 0 && pitch % 16 == 0 &&
                            (data_padded == nullptr || aligned16(data_padded));
  if (!rows_aligned && pitch == shard_size && (data_padded == nullptr || aligned16(data_padded)) &&
      aligned16(shards)) {
    // rows at any byte offset, back to back: the data rows are one flat copy and
    // the parity row one XOR pass over windows of them -- a single launch
    RowCopyXor r;
    const char* src = data_padded ? reinterpret_cast<const char*>(data_padded) : reinterpret_cast<const char*>(shards);
    if (data_padded) {
      r.src = src;
      r.dst = reinterpret_cast<char*>(shards);
      r.copy_len = (int64_t)data_shards * shard_size;
    }
    r.nin = data_shards;
    for (int i = 0; i < data_shards; ++i) r.in[i] = src + (int64_t)i * shard_size;
    r.out0 = reinterpret_cast<char*>(shards) + (int64_t)data_shards * shard_size;
    r.len = shard_size;
    return run_row_copy_xor(r, s);
  }
  if (data_padded) {
    int rc = rows_pack(data_padded, (int64_t)data_shards * shard_size, nullptr, 0, shards, pitch, shard_size,
                       data_shards, s);
    if (rc) return rc;
  }
  LinearPass a{};
  a.field = Field::XOR;
  a.split = INT64_MAX;
  a.begin = 0;
  a.end = shard_size;
  for (int r = 0; r < data_shards; ++r) set_row_in(a, reinterpret_cast<const char*>(shards), pitch, r);
  set_row_out(a, reinterpret_cast<char*>(shards) + (int64_t)data_shards * pitch, shard_size);
  return run_linear(a, s);
}

int gsec_xor_reconstruct(uint8_t* shards, uint8_t* recovered_missing, int64_t shard_size, int64_t pitch,
                         int32_t data_shards, const int32_t* missing, int32_t missing_count, gsec_stream_t stream) {
  GSEC_REQUIRE(shards != nullptr, "shards is null");
  GSEC_REQUIRE(data_shards >= 1 && data_shards <= kLinMaxIn, "data_shards=%d must be in [1, %d]", data_shards,
               kLinMaxIn);
  GSEC_REQUIRE(shard_size >= 1 && pitch >= shard_size, "bad shard_size/pitch");
  // Like reconstruct_xor_kernel (benchmark/xor/kernel.cu:56-57, :63, :77): no
  // work unless exactly one index in [0, data_shards] is missing.
  if (missing_count != 1 || missing == nullptr) return GSEC_OK;
  const int miss = missing[0];
  if (miss < 0 || miss > data_shards) return GSEC_OK;
  LinearPass a{};
  a.field = Field::XOR;
  a.split = INT64_MAX;
  a.begin = 0;
  a.end = shard_size;
  const char* base = reinterpret_cast<const char*>(shards);
  for (int r = 0; r <= data_shards; ++r)
    if (r != miss) set_row_in(a, base, pitch, r);
  set_row_out(a, reinterpret_cast<char*>(shards) + (int64_t)miss * pitch, shard_size);
  if (recovered_missing) set_row_out(a, reinterpret_cast<char*>(recovered_missing), shard_size);
  return run_linear(a, as_stream(stream));
}

// --------------------------------------------------------- RDP-ref compat ---
int gsec_rdpref_pack_row(const uint16_t* k_blk, const uint16_t* v_blk, int64_t words, uint16_t* shards,
                         int64_t pitch_words, int32_t row, gsec_stream_t stream) {
  GSEC_REQUIRE(shards != nullptr && row >= 0, "bad shards/row");
  GSEC_REQUIRE(words >= 0 && pitch_words >= 2 * words, "shard_size must be >= 2 * words");
  if (words == 0) return GSEC_OK;
  return rows_pack(k_blk, 2 * words, v_blk, 2 * words, shards + (int64_t)row * pitch_words, 4 * words, 4 * words, 1,
                   as_stream(stream));
}

int gsec_rdpref_parity(uint16_t* rows, int64_t pitch_words, int32_t nd, int64_t S, int32_t star_base,
                       gsec_stream_t stream) {
  return rdpref_parity(rows, pitch_words, nd, S, star_base, as_stream(stream));
}

int gsec_rdpref_backup(const uint16_t* k_tn, const uint16_t* v_tn, uint16_t* shards, int64_t pitch_words,
                       int32_t nd, int64_t S, int64_t T, int64_t n, int32_t star_base, gsec_stream_t stream) {
  GSEC_REQUIRE(shards && nd >= 1 && S >= 1 && T >= 0 && n >= 0, "bad arguments");
  GSEC_REQUIRE((int64_t)nd * S >= 2 * T * n, "nd * S < 2 * T * n");
  const cudaStream_t s = as_stream(stream);
  int rc = rows_pack(k_tn, 2 * T * n, v_tn, 2 * T * n, shards, 2 * pitch_words, 2 * S, nd, s);
  if (rc) return rc;
  return rdpref_parity(shards, pitch_words, nd, S, star_base, s);
}

int gsec_rdpref_backup_bhtd(const uint16_t* k, const uint16_t* v, int64_t B, int64_t H, int64_t T, int64_t D,
                            uint16_t* shards, int64_t pitch_words, int32_t nd, int64_t S, int32_t star_base,
                            gsec_stream_t stream) {
  const cudaStream_t s = as_stream(stream);
  int rc = bhtd_pack(k, v, B, H, T, D, shards, pitch_words, nd, S, s);
  if (rc) return rc;
  return rdpref_parity(shards, pitch_words, nd, S, star_base, s);
}

namespace {
// The data row the reference recovery finally rewrites from P, or -1
// (benchmark/rdp/kernel.cu:402-507, see gsec.h).
int rdpref_target(int nd, int a, int b) {
  a = (a >= 0 && a < nd) ? a : -1;
  b = (b >= 0 && b < nd) ? b : -1;
  if (a >= 0 && b >= 0) return a != b ? (a < b ? a : b) : -1;
  if (a >= 0) return a;
  if (b >= 0) return b;
  return -1;
}
int rdpref_rebuild(uint16_t* shards, int64_t pitch_words, int nd, int64_t S, int target, cudaStream_t s) {
  if (target < 0) return GSEC_OK;
  LinearPass a{};
  a.field = Field::XOR;
  a.split = INT64_MAX;
  a.begin = 0;
  a.end = 2 * S;
  const char* base = reinterpret_cast<const char*>(shards);
  set_row_in(a, base, 2 * pitch_words, nd);  // P row
  for (int r = 0; r < nd; ++r)
    if (r != target) set_row_in(a, base, 2 * pitch_words, r);
  set_row_out(a, reinterpret_cast<char*>(shards + (int64_t)target * pitch_words), 2 * S);
  return run_linear(a, s);
}
}  // namespace

int gsec_rdpref_recovery(uint16_t* shards, int64_t pitch_words, uint16_t* out_tn, int32_t nd, int64_t S, int64_t T,
                         int64_t n, int32_t star_base, int32_t miss_a, int32_t miss_b, gsec_stream_t stream) {
  (void)star_base;  // only the overwritten provisional steps of the reference use it
  GSEC_REQUIRE(shards && out_tn && nd >= 1 && nd + 1 <= kLinMaxIn && S >= 1 && pitch_words >= S, "bad arguments");
  GSEC_REQUIRE((int64_t)nd * S >= 2 * T * n, "nd * S < 2 * T * n");
  const cudaStream_t s = as_stream(stream);
  if (pitch_words == S && S % 8 != 0 && aligned16(shards) && aligned16(out_tn)) {
    // rows back to back at any byte offset: the token stream is the first 4Tn
    // bytes of the rows, so one launch rebuilds the lost row in place (P and
    // the other rows read through windows), writes it into the stream too, and
    // copies the other rows' bytes of the stream
    const int target = rdpref_target(nd, miss_a, miss_b);
    const char* base = reinterpret_cast<const char*>(shards);
    const int64_t row = 2 * S;
    RowCopyXor r;
    r.src = base;
    r.dst = reinterpret_cast<char*>(out_tn);
    r.copy_len = 4 * T * n;
    if (target >= 0) {
      r.skip_lo = target * row;
      r.skip_hi = (target + 1) * row;
      for (int i = 0; i <= nd; ++i)
        if (i != target) r.in[r.nin++] = base + i * row;  // the other data rows and P (row nd)
      r.out0 = reinterpret_cast<char*>(shards) + target * row;
      r.out1 = reinterpret_cast<char*>(out_tn) + target * row;
      r.out1_len = r.copy_len - target * row;
      if (r.out1_len < 0) r.out1_len = 0;
      r.len = row;
    } else {
      r.nin = 1;  // nothing to rebuild: the copy alone
      r.in[0] = base;
    }
    return run_row_copy_xor(r, s);
  }
  int rc = rdpref_rebuild(shards, pitch_words, nd, S, rdpref_target(nd, miss_a, miss_b), s);
  if (rc) return rc;
  if (T * n == 0) return GSEC_OK;
  return rows_unpack(shards, 2 * pitch_words, 2 * S, nd, out_tn, 4 * T * n, nullptr, 0, s);
}

int gsec_rdpref_recovery_bhtd(uint16_t* shards, int64_t pitch_words, uint16_t* k_out, uint16_t* v_out, int64_t B,
                              int64_t H, int64_t T, int64_t D, int32_t nd, int64_t S, int32_t star_base,
                              int32_t miss_a, int32_t miss_b, gsec_stream_t stream) {
  (void)star_base;
  GSEC_REQUIRE(shards && nd >= 1 && nd + 1 <= kLinMaxIn && S >= 1 && pitch_words >= S, "bad arguments");
  const cudaStream_t s = as_stream(stream);
  int rc = rdpref_rebuild(shards, pitch_words, nd, S, rdpref_target(nd, miss_a, miss_b), s);
  if (rc) return rc;
  return bhtd_unpack(shards, pitch_words, nd, S, k_out, v_out, B, H, T, D, s);
}

// ------------------------------------------------------------ RS16 compat ---
int gsec_rs16_tables(uint16_t* gf_exp, uint16_t* gf_log) {
  GSEC_REQUIRE(gf_exp && gf_log, "null table pointer");
  const Gf16Tables& t = gf16t();
  memcpy(gf_exp, t.exp.data(), t.exp.size() * sizeof(uint16_t));
  memcpy(gf_log, t.log.data(), t.log.size() * sizeof(uint16_t));
  return GSEC_OK;
}

namespace {
// Run outputs in passes of two (the GF16 kernel packs two products per entry).
int rs16_passes(LinearPass base, const std::vector<char*>& outs, const std::vector<std::vector<uint16_t>>& coef,
                int64_t end, cudaStream_t s) {
  for (size_t j0 = 0; j0 < outs.size(); j0 += 2) {
    LinearPass a = base;
    a.nout = 0;
    for (size_t j = j0; j < outs.size() && j < j0 + 2; ++j) {
      for (int i = 0; i < a.nin; ++i) a.coef[a.nout][i] = coef[j][i];
      set_row_out(a, outs[j], end);
    }
    int rc = run_linear(a, s);
    if (rc) return rc;
  }
  return GSEC_OK;
}
}  // namespace

int gsec_rs16_encode(const uint16_t* data_padded, uint16_t* shards, int64_t pitch_words, int32_t data_shards,
                     int32_t parity_shards, int64_t shard_size, gsec_stream_t stream) {
  GSEC_REQUIRE(shards != nullptr, "shards is null");
  GSEC_REQUIRE(data_shards >= 1 && data_shards <= kLinMaxIn, "data_shards=%d must be in [1, %d]", data_shards,
               kLinMaxIn);
  GSEC_REQUIRE(parity_shards >= 0, "parity_shards must be >= 0");
  GSEC_REQUIRE(shard_size >= 1 && pitch_words >= shard_size, "bad shard_size/pitch");
  const cudaStream_t s = as_stream(stream);
  const int64_t row_bytes = 2 * shard_size, pitch = 2 * pitch_words;
  if (data_padded) {
    int rc = rows_pack(data_padded, (int64_t)data_shards * row_bytes, nullptr, 0, shards, pitch, row_bytes,
                       data_shards, s);
    if (rc) return rc;
  }
  if (parity_shards == 0) return GSEC_OK;
  LinearPass a{};
  a.field = Field::GF16;
  a.split = INT64_MAX;
  a.begin = 0;
  a.end = row_bytes;
  for (int r = 0; r < data_shards; ++r) set_row_in(a, reinterpret_cast<const char*>(shards), pitch, r);
  std::vector<char*> outs;
  std::vector<std::vector<uint16_t>> coef;
  for (int p = 0; p < parity_shards; ++p) {
    outs.push_back(reinterpret_cast<char*>(shards) + (int64_t)(data_shards + p) * pitch);
    std::vector<uint16_t> row(data_shards);
    // coef = gf_exp[((p + 1) * k) % GF_ORDER], benchmark/rs/kernel.cu:88-95
    for (int i = 0; i < data_shards; ++i) row[i] = gf16_exp(((p + 1) * i) % 65535);
    coef.push_back(row);
  }
  return rs16_passes(a, outs, coef, row_bytes, s);
}

int gsec_rs16_reconstruct(uint16_t* shards, int64_t pitch_words, int64_t shard_size, int32_t data_shards,
                          int32_t parity_shards, const int32_t* missing_data, int32_t nmiss,
                          const int32_t* parity_used, gsec_stream_t stream) {
  GSEC_REQUIRE(shards != nullptr, "shards is null");
  GSEC_REQUIRE(data_shards >= 1 && parity_shards >= 0, "bad shard counts");
  GSEC_REQUIRE(shard_size >= 1 && pitch_words >= shard_size, "bad shard_size/pitch");
  GSEC_REQUIRE(nmiss >= 0 && nmiss <= 16, "m (missing data shards) must be <= 16");
  if (nmiss == 0) return GSEC_OK;
  GSEC_REQUIRE(missing_data && parity_used, "null index arrays");
  GSEC_REQUIRE(data_shards <= kLinMaxIn, "data_shards=%d must be <= %d", data_shards, kLinMaxIn);
  std::vector<bool> miss(data_shards, false);
  for (int c = 0; c < nmiss; ++c) {
    GSEC_REQUIRE(missing_data[c] >= 0 && missing_data[c] < data_shards && !miss[missing_data[c]],
                 "missing data index %d invalid or repeated", missing_data[c]);
    miss[missing_data[c]] = true;
    GSEC_REQUIRE(parity_used[c] >= 0 && parity_used[c] < parity_shards, "parity index %d invalid", parity_used[c]);
  }
  const int m = nmiss;
  // V[r][c] = gf_exp[((pused[r]+1) * missing[c]) % 65535] and its Gauss-Jordan
  // inverse, step for step as benchmark/rs/kernel.cu:135-185 (singular columns
  // are skipped the same way).
  std::vector<uint16_t> V((size_t)m * m), inv((size_t)m * m);
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < m; ++c) V[(size_t)r * m + c] = gf16_exp(((parity_used[r] + 1) * missing_data[c]) % 65535);
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < m; ++c) inv[(size_t)r * m + c] = r == c ? 1 : 0;
  for (int i = 0; i < m; ++i) {
    int pr = i;
    while (pr < m && V[(size_t)pr * m + i] == 0) ++pr;
    if (pr == m) continue;
    if (pr != i)
      for (int c = 0; c < m; ++c) {
        std::swap(V[(size_t)i * m + c], V[(size_t)pr * m + c]);
        std::swap(inv[(size_t)i * m + c], inv[(size_t)pr * m + c]);
      }
    const uint16_t piv = V[(size_t)i * m + i];
    if (piv == 0) continue;
    const uint16_t ip = gf16_div_tab(1, piv);
    for (int c = 0; c < m; ++c) {
      V[(size_t)i * m + c] = gf16_mul_tab(V[(size_t)i * m + c], ip);
      inv[(size_t)i * m + c] = gf16_mul_tab(inv[(size_t)i * m + c], ip);
    }
    for (int r = 0; r < m; ++r) {
      if (r == i) continue;
      const uint16_t f = V[(size_t)r * m + i];
      if (!f) continue;
      for (int c = 0; c < m; ++c) {
        V[(size_t)r * m + c] ^= gf16_mul_tab(f, V[(size_t)i * m + c]);
        inv[(size_t)r * m + c] ^= gf16_mul_tab(f, inv[(size_t)i * m + c]);
      }
    }
  }
  // x_c = sum_r inv[c][r] * (P_r ^ sum_{k survives} a(r,k) D_k): one linear pass
  // over the used parity rows and the surviving data rows (field arithmetic
  // is exact, so folding the two steps gives the same words).
  const int64_t row_bytes = 2 * shard_size, pitch = 2 * pitch_words;
  const char* base = reinterpret_cast<const char*>(shards);
  LinearPass a{};
  a.field = Field::GF16;
  a.split = INT64_MAX;
  a.begin = 0;
  a.end = row_bytes;
  std::vector<int> cols;  // input c: parity (>= 0 -> row data_shards + pu) or data row
  for (int r = 0; r < m; ++r) set_row_in(a, base, pitch, data_shards + parity_used[r]);
  std::vector<int> surv;
  for (int kk = 0; kk < data_shards; ++kk)
    if (!miss[kk]) {
      set_row_in(a, base, pitch, kk);
      surv.push_back(kk);
    }
  std::vector<char*> outs;
  std::vector<std::vector<uint16_t>> coef;
  for (int c = 0; c < m; ++c) {
    std::vector<uint16_t> row(a.nin, 0);
    for (int r = 0; r < m; ++r) row[r] = inv[(size_t)c * m + r];
    for (size_t t = 0; t < surv.size(); ++t) {
      uint16_t acc = 0;
      for (int r = 0; r < m; ++r)
        acc ^= gf16_mul_tab(inv[(size_t)c * m + r], gf16_exp(((parity_used[r] + 1) * surv[t]) % 65535));
      row[m + t] = acc;
    }
    coef.push_back(row);
    outs.push_back(reinterpret_cast<char*>(shards) + (int64_t)missing_data[c] * pitch);
  }
  return rs16_passes(a, outs, coef, row_bytes, as_stream(stream));
}

// ------------------------------------------------------------------- IPC ----
namespace {
typedef CUresult (*GetRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(p);
  });
  return fn;
}
std::mutex g_ipc_mu;
std::map<std::pair<int, std::string>, void*> g_ipc_maps;  // (device, handle bytes) -> mapped base
}  // namespace

int gsec_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  GSEC_REQUIRE(ptr && handle && offset, "null argument");
  GetRangeFn fn = get_range_fn();
  if (!fn) {
    set_error("cuMemGetAddressRange is unavailable");
    return GSEC_ECUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("cuMemGetAddressRange failed for %p", ptr);
    return GSEC_ECUDA;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return GSEC_ECUDA;
  }
  static_assert(sizeof(h) == GSEC_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return GSEC_OK;
}

int gsec_ipc_import(const void* handle, int64_t offset, void** ptr) {
  GSEC_REQUIRE(handle && ptr && offset >= 0, "bad argument");
  int dev = 0;
  cudaGetDevice(&dev);
  const std::string key(static_cast<const char*>(handle), GSEC_IPC_HANDLE_BYTES);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  auto it = g_ipc_maps.find({dev, key});
  void* base = nullptr;
  if (it != g_ipc_maps.end()) {
    base = it->second;
  } else {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
      return GSEC_ECUDA;
    }
    g_ipc_maps[{dev, key}] = base;
  }
  *ptr = static_cast<char*>(base) + offset;
  return GSEC_OK;
}

int gsec_ipc_close_all(void) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  int rc = GSEC_OK;
  for (auto it = g_ipc_maps.begin(); it != g_ipc_maps.end();) {
    if (it->first.first == dev) {
      if (cudaIpcCloseMemHandle(it->second) != cudaSuccess) rc = GSEC_ECUDA;
      it = g_ipc_maps.erase(it);
    } else {
      ++it;
    }
  }
  if (rc) set_error("cudaIpcCloseMemHandle failed");
  return rc;
}

}  // extern "C"
