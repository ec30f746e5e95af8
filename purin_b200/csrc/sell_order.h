// Bank-aware internal row/column orders for the sliced-ELL gathers (host code).
//
// In the forward kernel a warp owns 32 lines (rows or columns) and, at step k,
// each lane gathers the iterate at the internal position of its line's k-th
// entry from shared memory.  A shared-memory request is served in one pass per
// group of lanes whose addresses fall in distinct banks: 8-byte loads are
// served per half-warp (16 lanes, position mod 16 picks the bank pair),
// 16-byte loads per quarter-warp (8 lanes, position mod 8), 4-byte loads per
// warp (position mod 32).  Lanes of a group that hit the same bank at
// different addresses take extra passes, and random sparsity makes that the
// common case.
//
// Lines of equal length can trade internal positions without changing any
// slice width or any arithmetic (each line's entries keep their order), so the
// orders are chosen by a local search over such swaps that minimises the
// passes of every gather step in both products (K y over rows, K^T lambda over
// columns).  The search is deterministic (fixed seed and move budget).
#pragma once

#include <cstdint>
#include <vector>

namespace purin {

struct BankOrderStats {
  int64_t passes_before = 0;  // model passes of one iteration's gathers (all levels)
  int64_t passes_after = 0;
  int64_t moves = 0;
  int64_t accepted = 0;
};

// row_order (m entries) and col_order (n entries) map an internal position to a
// line and are sorted by line length, descending; on return each is permuted
// within its runs of equal length.  Rows are given in CSR (r_ptr, r_col), columns
// in CSC (c_ptr, c_row) with entries in the order the kernel accumulates them.
// elem_bytes is the iterate's element size (4 or 8); the search minimises the
// passes of the one- and two-sample tiles' gathers, or with wide_tiles only those
// of the 16-byte gathers of the wide multi-sample tiles (quarter-warps, position
// mod 8).  max_moves caps the search.
BankOrderStats bank_aware_orders(int m, int n, const std::vector<int32_t>& r_ptr,
                                 const std::vector<int32_t>& r_col, const std::vector<int32_t>& c_ptr,
                                 const std::vector<int32_t>& c_row, int elem_bytes, bool wide_tiles,
                                 int64_t max_moves, std::vector<int>& row_order,
                                 std::vector<int>& col_order);

}  // namespace purin
