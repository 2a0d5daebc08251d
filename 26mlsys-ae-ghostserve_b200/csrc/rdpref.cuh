// rdpref.cuh — the reference's mod-S row/diagonal parity (see rdpref.cu).
#pragma once

#include "common.cuh"

namespace gsec {

struct RdpRefParityArgs {
  uint16_t* rows;     // [(nd + 2) rows] x pitch words; rows nd, nd+1 receive P, Q
  int64_t pitch;      // words between rows
  int64_t S;          // words per row
  int64_t excl[32];   // per data row: skipped Q position, -1 for none
  int nd;
  bool vec_ok;        // rows 16-byte aligned and pitch a multiple of 8 words
};

int rdpref_parity(uint16_t* rows, int64_t pitch, int nd, int64_t S, int star_base, cudaStream_t s);

}  // namespace gsec
