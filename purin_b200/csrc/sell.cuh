// Sliced-ELL (SELL-32-sigma) views of the kept-row operator K and of K.T, in the
// kernels' internal row and column orders.
//
// Rows (for K @ x) and columns (for K.T @ y) are sorted by their number of
// nonzeros (descending, stable) and grouped in slices of 32 consecutive sorted
// lines; slice s stores its entries slot-major at ptr[s] + k * 32 + lane for
// k < width(s), so a warp whose lanes each own one line of the slice reads 32
// consecutive entries per step.  The sorted order is also the kernels' internal
// order: internal column position p holds external variable c_perm[p], internal
// row position q holds kept row r_perm[q] (-1 marks the padding positions that
// complete the last slice), and the entries' indices are internal positions.
// Per-sample vectors are permuted into these orders once per call so every
// per-iteration access is coalesced.  Entries past a line's length are
// padding: index = the extra zero element at position n_pos (or m_pos) of the
// gathered vector, value 0, so they add exact zeros after the line's real
// terms.  Within a line entries keep their original order (CSR order for rows;
// ascending row, i.e. the reference scatter's update order, for columns), so
// sums round exactly as the reference's sequential accumulation.
//
// When every internal position fits in 16 bits (idx16), the indices are also
// stored in pairs: the 32-bit word at ptr[s] + (k / 2) * 32 + lane, for even k,
// holds the positions of steps k (low half) and k + 1 (high half; the padding
// position when k + 1 == width(s)), so a warp reads the indices of two steps
// in one 128-byte request.  Only the first half of each slice's word range is
// used, which keeps the word index a function of ptr[s] alone.
#pragma once

#include <stdint.h>

namespace purin {

struct SellView {
  int C;                 // slice height (32)
  int nsl_r, nsl_c;      // slices
  int nnz_r, nnz_c;      // stored entries (with padding)
  int m_pos, n_pos;      // internal row / column positions (nsl * 32)
  const int* r_ptr;      // nsl_r + 1 entry offsets
  const int* r_perm;     // m_pos: kept row of each internal row position, -1 for padding
  const int* r_idx;      // nnz_r: internal column position, n_pos for padding
  const int* r_slot;     // nnz_r: kept CSR slot, -1 for padding
  const int* c_ptr;      // nsl_c + 1
  const int* c_perm;     // n_pos: variable of each internal column position, -1 for padding
  const int* c_idx;      // nnz_c: internal row position, m_pos for padding
  const int* c_slot;     // nnz_c: kept CSR slot, -1 for padding
  int idx16;                  // 1: r_idx2 / c_idx2 are present
  const uint32_t* r_idx2;     // nnz_r words: r_idx in pairs of steps (see above)
  const uint32_t* c_idx2;     // nnz_c words: c_idx in pairs of steps
};

}  // namespace purin
