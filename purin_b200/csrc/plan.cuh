// Device-resident sparse structure of a prepared CP projection.
//
// Built once per plan (PreparedChambollePockProjection.__post_init__,
// src/purin/solvers/chambolle_pock/solver.py:32-65).  The reference keeps a
// padded ELL layout (kernels.py:26-40) and performs K.T products as scatters
// (linalg/sparse/operators.py:521-533); here the same pattern is stored as CSR
// for K @ x and as CSC (entries sorted by row, i.e. the scatter's update order)
// for K.T @ y, so both products are gathers with deterministic summation order.
#pragma once

#include <stdint.h>

#include <vector>

#include "sell.cuh"

#include "../../include/purin_cp.h"

namespace purin {

struct DevStructure {
  int n;
  int me;
  int m;       // kept rows: me + kept inequality rows
  int nnz;     // kept nonzeros
  // Kept rows (the CP operator K).
  const int* row_ptr;   // m + 1
  const int* col;       // nnz
  const int* col_ptr;   // n + 1
  const int* csc_row;   // nnz, kept row index, ascending per column
  const int* csc_slot;  // nnz, kept CSR slot
  // All public rows (post-processing).
  int m_all;
  int nnz_all;
  const int* row_ptr_all;
  const int* col_all;
  const int* col_ptr_all;
  const int* csc_row_all;
  const int* csc_slot_all;
  const int* kept_rows;   // m: public row index
  const int* kept_slots;  // nnz: public CSR slot
  // Bound rows (singleton inequalities turned into box bounds).
  int n_bound;
  const int* bound_rows;
  const int* bound_slot;
  const int* bound_var;
  const int* var_bound_ptr;   // n + 1
  const int* var_bound_list;  // n_bound, bound index k per variable
};

}  // namespace purin

// Forward tile shapes the planner considers (capi.cu's shape table).
constexpr int kForwardShapeCount = 13;

// A structure whose stored entries (value plus 16-bit index, both products)
// exceed 384 KB streams from L2 once per tile-iteration; the forward then uses
// wide multi-sample tiles (16-byte gathers per lane), and the bank-aware line
// order is chosen for those gathers.
inline bool wide_structure(int64_t kept_nnz, size_t elem_bytes) {
  return (size_t)(2 * kept_nnz) * (elem_bytes + sizeof(uint16_t)) > (384u << 10);
}

struct PurinCpPlan {
  PurinCpPlanInfo info;
  purin::DevStructure dev;
  void* device_block = nullptr;  // one cudaMalloc holding every index array
  // Host copies for purin_cp_plan_indices.
  std::vector<int32_t> kept_rows, kept_slots, bound_rows, bound_slots, bound_vars;
  std::vector<int32_t> kept_row_ptr, kept_cols;
  int sm_count = 0;
  int max_smem_optin = 0;
  // Sliced-ELL layout (C = 32) in the internal row/column orders, built at creation.
  purin::SellView sell[1];
  void* sell_block = nullptr;
  // Resident forward CTAs per SM by [diagonal steps][shared values][tile shape]
  // (-1: not queried yet); filled on first use, the same value by any thread.
  // [distance | distance + diagonal steps | QP | QP with per-variable coefficients]
  // x [per-sample values | shared values] x tile shape
  int fwd_blocks[4][2][kForwardShapeCount];

  PurinCpPlan() {
    for (auto& a : fwd_blocks)
      for (auto& b : a)
        for (int& c : b) c = -1;
  }
};
