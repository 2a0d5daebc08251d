// layout.cuh — KV tensors <-> shard rows (see layout.cu).
#pragma once

#include "common.cuh"

namespace gsec {

int rows_pack(const void* s0, int64_t len0, const void* s1, int64_t len1, void* rows, int64_t pitch,
              int64_t row_bytes, int nrows, cudaStream_t s);
int rows_unpack(const void* rows, int64_t pitch, int64_t row_bytes, int nrows, void* d0, int64_t len0, void* d1,
                int64_t len1, cudaStream_t s);
// pitch and S in u16 words.
int bhtd_pack(const uint16_t* k, const uint16_t* v, int64_t B, int64_t H, int64_t T, int64_t D, uint16_t* rows,
              int64_t pitch, int nd, int64_t S, cudaStream_t s);
int bhtd_unpack(const uint16_t* rows, int64_t pitch, int nd, int64_t S, uint16_t* k, uint16_t* v, int64_t B,
                int64_t H, int64_t T, int64_t D, cudaStream_t s);

// Pool rows by slot index (gather: pool -> buf, scatter: buf -> pool); see layout.cu.
int slots_move(bool gather, void* const* pools, int npools, int64_t pitch, int64_t plane, int nplanes,
               int64_t row_bytes, const void* slots, int slot_bytes, int64_t n, int64_t pool_rows, void* lo,
               void* hi, int64_t split, cudaStream_t s);
// Status word of the slot kernels (bit 0: a slot past the pool's rows).
int copy_gather(const void* const* src, const int64_t* bytes, int n, void* dst, cudaStream_t s);
unsigned layout_device_status(bool clear);
// Status word of the gather kernel (bit 0: a bounded wait gave up).
unsigned gather_device_status(bool clear);

}  // namespace gsec
