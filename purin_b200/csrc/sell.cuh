// Sliced-ELL (SELL-C-sigma) views of the kept-row operator K and of K.T.
//
// Rows (for K @ x) and columns (for K.T @ y) are sorted by their number of
// nonzeros (descending, stable) and grouped in slices of C consecutive sorted
// rows; slice s stores its entries slot-major at ptr[s] + k * C + lane for
// k < width(s).  A warp whose C lane-groups each own one row of the slice
// therefore reads C consecutive entries per step (coalesced), and the slice
// width bounds the per-row loop.  Entries past a row's length are padding:
// index = the padded element of the gathered vector (always zero) and
// value 0, so they add exact zeros after the row's real terms.  Within a row
// entries keep their original order (CSR order for rows; ascending row, i.e.
// the reference scatter's update order, for columns), so sums round exactly
// as the reference's sequential accumulation.
#pragma once

#include <stdint.h>

namespace purin {

struct SellView {
  int C;
  int nsl_r, nsl_c;      // slices
  int nnz_r, nnz_c;      // stored entries (with padding)
  const int* r_ptr;      // nsl_r + 1 entry offsets
  const int* r_perm;     // nsl_r * C: kept row of each sorted position, -1 for padding rows
  const int* r_idx;      // nnz_r: column index, n for padding
  const int* r_slot;     // nnz_r: kept CSR slot, -1 for padding
  const int* c_ptr;      // nsl_c + 1
  const int* c_perm;     // nsl_c * C: column of each sorted position, -1 for padding
  const int* c_idx;      // nnz_c: kept row index, m for padding
  const int* c_slot;     // nnz_c: kept CSR slot, -1 for padding
};

}  // namespace purin
