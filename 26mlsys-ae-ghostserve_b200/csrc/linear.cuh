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
  uint32_t unity = 1;  // always 1; read from the launch parameters, so the compiler cannot fold it
};

// Device status word of the staged linear kernels (non-zero: a bounded wait gave up).
unsigned linear_device_status(bool clear);

// Launch one pass on `stream` (chooses vector or scalar kernels by alignment).
int run_linear(const LinearPass& pass, cudaStream_t stream);

}  // namespace gsec
