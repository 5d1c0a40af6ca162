// Index arithmetic of the distributed 2D transform, shared by dist.cu and the
// CPU emulator in the test suite.
//
// P ranks, B = N/P. Layouts of rank r's share of an N x N image:
//   row slab    rows [r*B, r*B + B), row-major B x N;
//   column slab columns [r*B, r*B + B) of all N rows, row-major N x B;
//   blocked     the row pass's output, [q][row][col] with B x B blocks, block
//               q holding columns [q*B, q*B + B) of this rank's rows.
// Both exchanges move, for a chunk of rows [r0, r1) of every B x B block,
//   send  src + q*B*B + r0*B   (to rank q)
//   recv  dst + p*B*B + r0*B   (from rank p)
// (r1 - r0) * B values each way. From a blocked buffer this builds the
// column slab (row p*B + r of the slab is row r of source p's block); from a
// column slab it builds [p][row][col] blocks that a gather turns into the
// row slab.
#pragma once

#include <stdint.h>

#include "plan.h"

namespace ferrum {

inline int64_t dist_block_offset(int64_t peer, int64_t r0, int64_t b) { return peer * b * b + r0 * b; }

// Rows [r0, r1) of chunk c out of `chunks` over b rows.
inline void dist_chunk(int64_t b, int chunks, int c, int64_t& r0, int64_t& r1) {
  r0 = b * c / chunks;
  r1 = b * (c + 1) / chunks;
}

inline int dist_chunks(int64_t b) { return b >= 4 ? 4 : (int)b; }

// Peer-memory path: element e of local row f of rank p lives in rank
// (e >> log_b)'s receive slab (its N x B column slab) at
// p*B*B + peer_offset(f, e, log_b), i.e. row p*B + f, column e mod B.
FERRUM_HD inline int64_t peer_offset(int64_t f, int64_t e, int log_b) {
  return (f << log_b) + (e & (((int64_t)1 << log_b) - 1));
}

}  // namespace ferrum
