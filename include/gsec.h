/*
 * gsec.h — C ABI of the B200 KV-cache erasure-coding engine (libgsec.so).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as an opaque pointer, 0 = legacy default stream), launches its
 * kernels on that stream and returns without synchronising.  Nothing here
 * allocates device memory; the caller owns every buffer.  Pointers to shards
 * may point into another GPU's memory once it has been mapped with
 * gsec_ipc_import (NVLink peer loads/stores).
 *
 * Return codes: GSEC_OK (0) or one of the GSEC_E* values below; the message of
 * the last failure on the calling thread is returned by gsec_last_error().
 *
 * Reference interfaces replaced are cited as file:line of the reference
 * project (GhostServe artifact); "ref-compat" entries reproduce the
 * reference's bytes exactly, "engine" entries are the B200-native codec that
 * the tensor-parallel hook uses.
 */
#ifndef GSEC_H_
#define GSEC_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GSEC_API __attribute__((visibility("default")))
#else
#define GSEC_API
#endif

typedef void* gsec_stream_t; /* a cudaStream_t */

enum {
  GSEC_OK = 0,
  GSEC_EINVAL = 1,          /* bad argument (shape, index, alignment, code parameters) */
  GSEC_EUNRECOVERABLE = 2,  /* erasure pattern cannot be decoded by this code */
  GSEC_ECUDA = 3,           /* a CUDA runtime call or kernel launch failed */
  GSEC_ETIMEOUT = 4,        /* a bounded device-side wait gave up */
  GSEC_EUNSUPPORTED = 5     /* parameters outside what this build implements */
};

enum {
  GSEC_SCHEME_XOR = 0, /* single parity, byte-wise XOR */
  GSEC_SCHEME_RDP = 1, /* Row-Diagonal Parity (Corbett et al., FAST'04), p prime, k <= p-1 */
  GSEC_SCHEME_RS8 = 2  /* Reed-Solomon over GF(2^8), poly 0x11d, Cauchy generator */
};

/* Parameters of one erasure code (engine entries). */
typedef struct gsec_code {
  int32_t scheme;  /* GSEC_SCHEME_* */
  int32_t k;       /* data shards (XOR: 1..32, RDP: 1..p-1, RS8: 1..32) */
  int32_t m;       /* parity shards (XOR: 1, RDP: 2, RS8: 1..4) */
  int32_t p;       /* RDP prime, 3..17 (ignored otherwise) */
  int64_t unit;    /* RDP stripe unit in bytes, multiple of 16 (ignored otherwise) */
} gsec_code;

/* ------------------------------------------------------------------------- */
/* Library                                                                    */
/* ------------------------------------------------------------------------- */

/* Message of the last failed call on this thread ("" if none). */
GSEC_API const char* gsec_last_error(void);
/* Library version string. */
GSEC_API const char* gsec_version(void);
/* Device status of the current GPU (synchronous: waits for this device's
 * pending work). Kernels that stage data through TMA bulk copies bound every
 * wait; one that gives up sets a bit here and returns early, so a non-zero
 * status means some call since the last clear produced incomplete output.
 * clear != 0 resets it. No counterpart in the reference (its kernels have no
 * waits). */
GSEC_API int gsec_device_status(uint32_t* status, int32_t clear);

/* ------------------------------------------------------------------------- */
/* Engine: position-sliced encode / decode over per-shard pointers            */
/* Replaces the gather + pack + parity sequence of the reference hook,        */
/* bench_ghostserve_rdp.py:303-360 (_distributed_gather_kv,                    */
/* _compute_parity_to_cpu), and the codec cores of                             */
/* benchmark/xor/kernel.cu:17-88, benchmark/rs/kernel.cu:67-222.               */
/* ------------------------------------------------------------------------- */

/* Bytes of one parity shard for data shards of data_bytes bytes
 * (RDP pads to whole stripes of (p-1)*unit bytes; XOR/RS8 do not pad). */
GSEC_API int gsec_parity_bytes(const gsec_code* code, int64_t data_bytes, int64_t* out_bytes);

/* Encode parity bytes [begin, end) of all m parity shards.
 *   data_lo[i], data_hi[i]: data shard i is the byte string
 *       data_lo[i][0 .. split) ++ data_hi[i][0 .. data_bytes-split)
 *     (pass data_hi = NULL, or split >= data_bytes, for one contiguous buffer;
 *      this lets the K and V halves of a rank's KV be one shard without a copy);
 *     bytes past data_bytes read as zero (RDP tail stripe).
 *   parity[j]: base of parity shard j (byte 0; only [begin, end) is written).
 *   data_bytes and split must be multiples of 16, every pointer 16-byte aligned;
 *   begin/end must be multiples of 16 (XOR/RS8) or of the stripe (RDP), except
 *   that end may equal gsec_parity_bytes(). Any pointer may be a mapped peer
 *   pointer (gsec_ipc_import). */
GSEC_API int gsec_encode(const gsec_code* code,
                const void* const* data_lo, const void* const* data_hi, int64_t split,
                int64_t data_bytes, void* const* parity,
                int64_t begin, int64_t end, gsec_stream_t stream);

/* Rebuild the erased shards over byte range [begin, end).
 *   shard_lo/shard_hi: k+m entries, data shards 0..k-1 then parity k..k+m-1,
 *     same split convention as gsec_encode (parity shards are contiguous:
 *     shard_hi entries for parity are ignored). Surviving shards are read,
 *     erased shards are written (data shards only up to data_bytes).
 *   erased: nerased distinct indices in [0, k+m); nerased <= m.
 * Returns GSEC_EUNRECOVERABLE for patterns the code cannot decode. */
GSEC_API int gsec_decode(const gsec_code* code,
                void* const* shard_lo, void* const* shard_hi, int64_t split,
                int64_t data_bytes, const int32_t* erased, int32_t nerased,
                int64_t begin, int64_t end, gsec_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Layout: [K | V] byte stream <-> shard rows (folds the reference pack /     */
/* unpack passes into one strided copy).                                       */
/* ------------------------------------------------------------------------- */

/* Copy the stream src0[0..len0) ++ src1[0..len1) into nrows rows of row_bytes
 * bytes (row r at rows + r*pitch), zero-filling past the stream end.
 * Replaces pack_kv (benchmark/xor/kernel.cu:93-119, :193-207) followed by the
 * zero-pad copy of benchmark/xor/main.py:89-90, and pack_fp16_pair_to_u16
 * (benchmark/rs/kernel.cu:36-49, :225-243) followed by benchmark/rs/main.py:104-108. */
GSEC_API int gsec_rows_pack(const void* src0, int64_t len0, const void* src1, int64_t len1,
                   void* rows, int64_t pitch, int64_t row_bytes, int32_t nrows,
                   gsec_stream_t stream);

/* Inverse of gsec_rows_pack: the first len0+len1 bytes of the row stream go to
 * dst0[0..len0) and dst1[0..len1). Replaces unpack_kv
 * (benchmark/xor/kernel.cu:122-146, :209-223) and u16_to_fp16_split
 * (benchmark/rs/kernel.cu:51-64, :245-263). */
GSEC_API int gsec_rows_unpack(const void* rows, int64_t pitch, int64_t row_bytes, int32_t nrows,
                     void* dst0, int64_t len0, void* dst1, int64_t len1,
                     gsec_stream_t stream);

/* Gather the rows of a slot list out of a KV pool [pool_rows, nplanes, ...]:
 * plane p (at byte offset p*plane inside a slot's pitch-byte record) of slot
 * slots[i] goes to dst + (p*n + i)*row_bytes. A negative slot gives a zero row
 * (no active count is needed on the host). slot_bytes = 4 or 8 (int32/int64
 * list). Pool, dst, pitch, plane and row_bytes 16-byte aligned. A slot >=
 * pool_rows zeroes its row and sets bit 16 of gsec_device_status.
 * Replaces the delta-KV extraction of the reference hook: the active count
 * read back to the host and kv_pool[active_slots, 0/1].contiguous()
 * (bench_ghostserve_rdp.py:449-458). */
GSEC_API int gsec_slots_gather(const void* pool, int64_t pitch, int64_t plane, int32_t nplanes,
                      int64_t row_bytes, const void* slots, int32_t slot_bytes, int64_t n,
                      int64_t pool_rows, void* dst, gsec_stream_t stream);
/* Inverse of gsec_slots_gather: src's rows back into the pool (rows of
 * negative slots are skipped). Used to restore a rebuilt delta into a
 * replacement rank's pool; the reference has no restore path. */
GSEC_API int gsec_slots_scatter(void* pool, int64_t pitch, int64_t plane, int32_t nplanes,
                       int64_t row_bytes, const void* slots, int32_t slot_bytes, int64_t n,
                       int64_t pool_rows, const void* src, gsec_stream_t stream);

/* One-kernel gather: dst = src[0][0..bytes[0]) ++ ... ++ src[n-1][0..bytes[n-1])
 * (n <= 32; every source, size and dst 16-byte aligned/multiple of 16). Sources
 * may be mapped peer buffers: this is a plain peer-read copy (bulk copies
 * through shared memory, no arithmetic), the copy the reference hook does with
 * two NCCL gathers to one rank (bench_ghostserve_rdp.py:303-332) done as reads
 * by the destination GPU; bench.py times it as the NVLink read ceiling of a
 * shard placement. A bounded wait that gives up sets bit 24 of
 * gsec_device_status. */
GSEC_API int gsec_copy_gather(const void* const* src, const int64_t* bytes, int32_t n, void* dst,
                              gsec_stream_t stream);

/* gsec_slots_gather over the same slot list in several pools at once (the
 * per-layer KV pools of one attention backend, npools <= 128, all of the same
 * geometry): pool q, plane p, list position i goes to byte
 * ((q*nplanes + p)*n + i)*row_bytes of the two-segment destination
 * dst_lo[0..split) ++ dst_hi[...] (dst_hi = NULL: one buffer). One launch
 * gathers a prefill chunk's delta KV of every layer, which the hook's
 * per-chunk mode encodes once instead of once per layer call; the reference
 * has no such mode (it encodes after every forward_extend call,
 * bench_ghostserve_rdp.py:424-471). */
GSEC_API int gsec_slots_gather_pools(void* const* pools, int32_t npools, int64_t pitch, int64_t plane,
                                     int32_t nplanes, int64_t row_bytes, const void* slots, int32_t slot_bytes,
                                     int64_t n, int64_t pool_rows, void* dst_lo, void* dst_hi, int64_t split,
                                     gsec_stream_t stream);
/* Inverse of gsec_slots_gather_pools (rows of negative slots are skipped). */
GSEC_API int gsec_slots_scatter_pools(void* const* pools, int32_t npools, int64_t pitch, int64_t plane,
                                      int32_t nplanes, int64_t row_bytes, const void* slots, int32_t slot_bytes,
                                      int64_t n, int64_t pool_rows, const void* src_lo, const void* src_hi,
                                      int64_t split, gsec_stream_t stream);

/* Stream-ordered copy of `bytes` bytes between any two addresses the device
 * can reach (device, pinned host, mapped peer). The hook offloads each parity
 * slice with it, one call per parity shard. No reference counterpart (the
 * reference copies P and Q with a blocking tensor .to("cpu"),
 * bench_ghostserve_rdp.py:362-366). */
GSEC_API int gsec_copy_async(void* dst, const void* src, int64_t bytes, gsec_stream_t stream);

/* ------------------------------------------------------------------------- */
/* ref-compat: XOR (benchmark/xor/kernel.cu)                                   */
/* ------------------------------------------------------------------------- */

/* encode_xor: shards rows 0..k-1 = data_padded rows, row k = XOR of them.
 * Rows of shard_size bytes at shards + r*pitch. Replaces encode_xor_launcher,
 * benchmark/xor/kernel.cu:158-171 (kernel :17-41). data_padded may be NULL when
 * the data rows are already in place in `shards` (parity only). */
GSEC_API int gsec_xor_encode(const uint8_t* data_padded, uint8_t* shards, int32_t data_shards,
                    int64_t shard_size, int64_t pitch, gsec_stream_t stream);

/* reconstruct_xor: rebuild the one missing row (data or parity) of `shards` in
 * place and also write it to recovered_missing (may be NULL). missing is a host
 * array. Replaces reconstruct_xor_launcher, benchmark/xor/kernel.cu:173-191
 * (kernel :47-88); the reference reads missing_indices from device memory. */
GSEC_API int gsec_xor_reconstruct(uint8_t* shards, uint8_t* recovered_missing, int64_t shard_size,
                         int64_t pitch, int32_t data_shards, const int32_t* missing,
                         int32_t missing_count, gsec_stream_t stream);

/* ------------------------------------------------------------------------- */
/* ref-compat: the reference's mod-S "RDP" (benchmark/rdp/kernel.cu and the    */
/* hook extension in bench_ghostserve_rdp.py:92-207), u16 words.               */
/* ------------------------------------------------------------------------- */

/* pack_row_from_block: row `row` of `shards` = [k_blk words | v_blk words].
 * Replaces bench_ghostserve_rdp.py:152-175 (kernel :105-118). */
GSEC_API int gsec_rdpref_pack_row(const uint16_t* k_blk, const uint16_t* v_blk, int64_t words,
                         uint16_t* shards, int64_t pitch_words, int32_t row,
                         gsec_stream_t stream);

/* compute_rdp_parity: P row (nd) = XOR of data rows, Q row (nd+1) = diagonal
 * XOR mod S skipping one star cell per row. Replaces
 * bench_ghostserve_rdp.py:181-199 (kernel :121-150) and the parity half of
 * fused_backup_full_kv_launcher, benchmark/rdp/kernel.cu:383-394 (kernel :76-107). */
GSEC_API int gsec_rdpref_parity(uint16_t* rows, int64_t pitch_words, int32_t nd, int64_t S,
                       int32_t star_base, gsec_stream_t stream);

/* fused_backup_full_kv: pack the token-major stream [K_TN | V_TN] (T*n words
 * each) into nd rows of S words and compute P/Q. Replaces
 * fused_backup_full_kv_launcher, benchmark/rdp/kernel.cu:366-395. */
GSEC_API int gsec_rdpref_backup(const uint16_t* k_tn, const uint16_t* v_tn, uint16_t* shards,
                       int64_t pitch_words, int32_t nd, int64_t S, int64_t T, int64_t n,
                       int32_t star_base, gsec_stream_t stream);

/* Same as gsec_rdpref_backup but reads K and V in their [B,H,T,D] layout and
 * applies the [T, B*H*D] permutation while packing (benchmark/rdp/main.py:66-67
 * does it as two .contiguous() copies). */
GSEC_API int gsec_rdpref_backup_bhtd(const uint16_t* k, const uint16_t* v, int64_t B, int64_t H,
                            int64_t T, int64_t D, uint16_t* shards, int64_t pitch_words,
                            int32_t nd, int64_t S, int32_t star_base, gsec_stream_t stream);

/* fused_recovery_full_kv: reproduce the reference recovery on `shards` in place
 * and write the token-major stream [K_TN | V_TN] to out_tn. Replaces
 * fused_recovery_full_kv_launcher, benchmark/rdp/kernel.cu:397-521. The
 * reference's two-erasure sequence ends with rebuild_row_from_P(a) then
 * rebuild_row_from_P(b) (:472-490), which leaves row b as it is and sets row
 * min(a,b) = P ^ (all other rows); this entry produces exactly those bytes. */
GSEC_API int gsec_rdpref_recovery(uint16_t* shards, int64_t pitch_words, uint16_t* out_tn,
                         int32_t nd, int64_t S, int64_t T, int64_t n, int32_t star_base,
                         int32_t miss_a, int32_t miss_b, gsec_stream_t stream);

/* As gsec_rdpref_recovery, but writes K and V back in [B,H,T,D] layout
 * (benchmark/rdp/main.py:121-124 does the inverse permutation as copies). */
GSEC_API int gsec_rdpref_recovery_bhtd(uint16_t* shards, int64_t pitch_words, uint16_t* k_out,
                              uint16_t* v_out, int64_t B, int64_t H, int64_t T, int64_t D,
                              int32_t nd, int64_t S, int32_t star_base, int32_t miss_a,
                              int32_t miss_b, gsec_stream_t stream);

/* ------------------------------------------------------------------------- */
/* ref-compat: Reed-Solomon over GF(2^16), poly 0x1100B (benchmark/rs)         */
/* ------------------------------------------------------------------------- */

/* init_gf_tables: exp (2*65535 entries) and log (65536 entries) tables, the
 * same values benchmark/rs/main.py:39-54 builds. Host memory. */
GSEC_API int gsec_rs16_tables(uint16_t* gf_exp, uint16_t* gf_log);

/* encode_rs_u16: rows 0..k-1 of `shards` = data_padded rows (skipped when
 * data_padded is NULL: data already in place), rows k..k+m-1 = parity
 * P_p = sum_i alpha^((p+1)*i mod 65535) * D_i. Replaces encode_rs_u16,
 * benchmark/rs/kernel.cu:265-285 (kernel :67-102). */
GSEC_API int gsec_rs16_encode(const uint16_t* data_padded, uint16_t* shards, int64_t pitch_words,
                     int32_t data_shards, int32_t parity_shards, int64_t shard_size,
                     gsec_stream_t stream);

/* reconstruct_rs_u16_inplace: rebuild the nmiss missing data rows from the
 * parity rows parity_used[0..nmiss) (host arrays). Replaces
 * reconstruct_rs_u16_inplace, benchmark/rs/kernel.cu:287-312 (kernel :105-222);
 * the m x m inversion is done once on the host with the same Gauss-Jordan
 * steps instead of once per thread block. */
GSEC_API int gsec_rs16_reconstruct(uint16_t* shards, int64_t pitch_words, int64_t shard_size,
                          int32_t data_shards, int32_t parity_shards,
                          const int32_t* missing_data, int32_t nmiss,
                          const int32_t* parity_used, gsec_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Peer mapping for the tensor-parallel path (CUDA IPC over NVLink)           */
/* Replaces the NCCL gathers of bench_ghostserve_rdp.py:321-331: peers' KV     */
/* is read in place by the encode kernel instead of being copied to one rank. */
/* ------------------------------------------------------------------------- */

#define GSEC_IPC_HANDLE_BYTES 64

/* Export the allocation containing ptr: 64-byte handle + ptr's offset in it. */
GSEC_API int gsec_ipc_export(const void* ptr, void* handle, int64_t* offset);
/* Map a peer allocation (current device) and return base + offset. Mapping the
 * same handle again returns the cached mapping. */
GSEC_API int gsec_ipc_import(const void* handle, int64_t offset, void** ptr);
/* Unmap every allocation mapped by gsec_ipc_import on the current device. */
GSEC_API int gsec_ipc_close_all(void);

#ifdef __cplusplus
}
#endif

#endif /* GSEC_H_ */
