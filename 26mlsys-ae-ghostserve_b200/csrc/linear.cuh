// linear.cuh — position-wise linear codes: every output shard byte (or u16
// word) at offset x is a GF-linear combination of the input shards' bytes at
// the same offset x.  Covers XOR parity and XOR rebuild, Reed-Solomon over
// GF(2^8) (encode and decode are both "outputs = matrix * inputs") and the
// reference's Reed-Solomon over GF(2^16).
#pragma once

#include "common.cuh"

namespace gsec {

constexpr int kLinMaxIn = 32;
constexpr int kLinMaxOut = 4;

enum class Field : int { XOR = 0, GF8 = 1, GF16 = 2 };

// One linear pass: outputs[j] = sum_i coef[j][i] * inputs[i] over [begin, end).
// A shard is the byte string lo[0..split) ++ hi[0..); contiguous shards pass
// hi = lo + split (so the select is an identity).
struct LinearPass {
  const char* in_lo[kLinMaxIn];
  const char* in_hi[kLinMaxIn];
  char* out_lo[kLinMaxOut];
  char* out_hi[kLinMaxOut];
  int64_t split;
  int64_t begin;      // byte offset, multiple of 16
  int64_t end;        // byte offset (may have a sub-16-byte tail)
  int64_t out_end[kLinMaxOut];  // an output is written only below this offset
  uint16_t coef[kLinMaxOut][kLinMaxIn];  // GF8 uses the low byte; XOR ignores
  int nin;
  int nout;
  Field field;
  int remote = 0;     // some input lies in another GPU's memory (read over NVLink)
};

// One launch that copies src[0..copy_len) to dst (bytes in [skip_lo, skip_hi)
// left to the XOR row) and writes one XOR row: out0[c] (and out1[c] for
// c < out1_len) = XOR_r in[r][c] for c in [0, len). src, dst and out1 - out0
// distance-compatible: src, dst 16-byte aligned, out1 with out0's alignment.
// The reference-layout calls whose shard rows start at any byte offset use it:
// encode_xor (data rows copied, parity row built) and the mod-S recovery
// (lost row rebuilt in place, all rows unpacked to the token stream).
struct RowCopyXor {
  const char* src = nullptr;
  char* dst = nullptr;
  int64_t copy_len = 0;
  int64_t skip_lo = 0, skip_hi = 0;
  const char* in[kLinMaxIn] = {};
  int nin = 0;
  char* out0 = nullptr;
  char* out1 = nullptr;
  int64_t out1_len = 0;
  int64_t len = 0;
};
int run_row_copy_xor(const RowCopyXor& a, cudaStream_t stream);

// Device status word of the staged linear kernels (non-zero: a bounded wait gave up).
unsigned linear_device_status(bool clear);

// Launch one pass on `stream` (chooses vector or scalar kernels by alignment).
int run_linear(const LinearPass& pass, cudaStream_t stream);

}  // namespace gsec
