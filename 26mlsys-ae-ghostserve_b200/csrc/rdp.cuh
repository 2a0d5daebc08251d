// rdp.cuh — textbook Row-Diagonal Parity kernels (see rdp.cu).
#pragma once

#include "common.cuh"

namespace gsec {

constexpr int kRdpMaxCols = 18;  // p + 1 columns for p <= 17

struct RdpEncodeArgs {
  const char* d_lo[16];
  const char* d_hi[16];
  char* parity[2];      // P and Q shard bases
  int64_t split;
  int64_t data_bytes;   // data shard bytes; reads at or past this offset are zero
  int64_t unit;         // stripe unit bytes (multiple of 16)
  int64_t s_begin, s_end;  // stripe range
  int k;
  int p;
  int remote = 0;       // some input lies in another GPU's memory (read over NVLink)
};

struct RdpDecodeArgs {
  const char* lo[kRdpMaxCols];  // indexed by column: 0..p-2 data, p-1 = P, p = Q
  const char* hi[kRdpMaxCols];
  char* out_lo[2];
  char* out_hi[2];
  uint32_t mask[2][16];  // per erased column and row: syndromes to XOR
  // The same solution as a straight-line program over the erased cells: step t
  // rebuilds cell (prog_out[t] >> 4 = erased column index, & 15 = row) as
  // (prog_chain[t] ? cell of step t-1 : 0) ^ XOR of the syndromes in prog_diff[t].
  uint32_t prog_diff[32];
  uint8_t prog_out[32];
  uint8_t prog_chain[32];
  int nprog;
  int out_col[2];
  int nout;
  uint32_t alive;        // bit c set: column c is read
  int64_t split;
  int64_t data_bytes;
  int64_t unit;
  int64_t s_begin, s_end;
  int p;
  int remote = 0;        // some input lies in another GPU's memory (read over NVLink)
};

bool rdp_prime_supported(int p);
// Device status word of the RDP kernels (non-zero: a bounded wait gave up).
unsigned rdp_device_status(bool clear);
int rdp_encode(const RdpEncodeArgs& a, cudaStream_t s);
int rdp_decode(const RdpDecodeArgs& a, cudaStream_t s);
int rdp_solve_masks(int p, const int* cols, int ncols, uint32_t mask[2][16]);
// Order the erased cells of a solved pattern into a chain program (fills
// prog_* and nprog of `a` from a.mask, a.nout and a.p).
void rdp_build_program(RdpDecodeArgs& a);

}  // namespace gsec
