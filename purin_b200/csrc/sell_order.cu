// Bank-aware internal orders for the sliced-ELL gathers (host code); the
// access model and the search are described in sell_order.h.
#include "sell_order.h"

#include <algorithm>
#include <random>

namespace purin {

namespace {

// Per (group of lanes, step) counts of gathered addresses per bank class.
struct Table {
  int group = 1, classes = 1, steps = 0, groups = 0;
  int group_shift = 0, class_mask = 0;  // group and classes are powers of two
  std::vector<uint8_t> count;   // [group][step][class] (a cell holds at most 32 lanes)
  std::vector<uint32_t> stamp;  // [group][step]: last move that touched the cell

  void init(int positions, int steps_, int group_, int classes_) {
    group = group_;
    classes = classes_;
    group_shift = 0;
    while ((1 << group_shift) < group) ++group_shift;
    class_mask = classes - 1;
    steps = steps_;
    groups = (positions + group - 1) / group;
    count.assign((size_t)groups * steps * classes, 0);
    stamp.assign((size_t)groups * steps, 0);
  }
  int cell(int pos, int step) const { return (pos >> group_shift) * steps + step; }
  int cls(int pos) const { return pos & class_mask; }
  int passes(int c) const {
    const uint8_t* v = &count[(size_t)c * classes];
    uint8_t best = 0;
    for (int b = 0; b < classes; ++b) best = v[b] > best ? v[b] : best;
    return best;
  }
  int64_t total() const {
    int64_t t = 0;
    for (int c = 0; c < groups * steps; ++c) t += passes(c);
    return t;
  }
  uint8_t& at(int c, int b) { return count[(size_t)c * classes + b]; }
};

struct Change {
  Table* t;
  int cell, cls, delta;
};

}  // namespace

BankOrderStats bank_aware_orders(int m, int n, const std::vector<int32_t>& r_ptr,
                                 const std::vector<int32_t>& r_col, const std::vector<int32_t>& c_ptr,
                                 const std::vector<int32_t>& c_row, int elem_bytes, bool wide_tiles,
                                 int64_t max_moves,
                                 std::vector<int>& row_order, std::vector<int>& col_order) {
  BankOrderStats stats;
  if (m <= 0 || n <= 0) return stats;
  auto rlen = [&](int r) { return r_ptr[r + 1] - r_ptr[r]; };
  auto clen = [&](int c) { return c_ptr[c + 1] - c_ptr[c]; };
  int rsteps = 0, csteps = 0;
  for (int r = 0; r < m; ++r) rsteps = std::max(rsteps, rlen(r));
  for (int c = 0; c < n; ++c) csteps = std::max(csteps, clen(c));
  if (rsteps == 0 || csteps == 0) return stats;

  // (c, j): row r is entry j of column c; (r, k): column c is entry k of row r.
  std::vector<int32_t> rent_ptr(m + 1, 0), cent_ptr(n + 1, 0);
  for (int c = 0; c < n; ++c)
    for (int e = c_ptr[c]; e < c_ptr[c + 1]; ++e) ++rent_ptr[c_row[e] + 1];
  for (int r = 0; r < m; ++r) rent_ptr[r + 1] += rent_ptr[r];
  std::vector<int32_t> rent_c(rent_ptr[m]), rent_j(rent_ptr[m]);
  {
    std::vector<int32_t> fill(rent_ptr.begin(), rent_ptr.end() - 1);
    for (int c = 0; c < n; ++c)
      for (int e = c_ptr[c]; e < c_ptr[c + 1]; ++e) {
        const int r = c_row[e];
        rent_c[fill[r]] = c;
        rent_j[fill[r]++] = e - c_ptr[c];
      }
  }
  for (int r = 0; r < m; ++r)
    for (int e = r_ptr[r]; e < r_ptr[r + 1]; ++e) ++cent_ptr[r_col[e] + 1];
  for (int c = 0; c < n; ++c) cent_ptr[c + 1] += cent_ptr[c];
  std::vector<int32_t> cent_r(cent_ptr[n]), cent_k(cent_ptr[n]);
  {
    std::vector<int32_t> fill(cent_ptr.begin(), cent_ptr.end() - 1);
    for (int r = 0; r < m; ++r)
      for (int e = r_ptr[r]; e < r_ptr[r + 1]; ++e) {
        const int c = r_col[e];
        cent_r[fill[c]] = r;
        cent_k[fill[c]++] = e - r_ptr[r];
      }
  }

  std::vector<int> rpos(m), cpos(n);
  for (int p = 0; p < m; ++p) rpos[row_order[p]] = p;
  for (int p = 0; p < n; ++p) cpos[col_order[p]] = p;

  // Access levels: the tile widths S = 1 and S = 2 (element of S values per
  // lane), or the 16-byte gathers of the wide tiles alone.
  const int nl = wide_tiles ? 1 : 2;
  int level_group[2] = {elem_bytes == 8 ? 16 : 32, elem_bytes == 8 ? 8 : 16};
  if (wide_tiles) level_group[0] = 8;
  std::vector<Table> rowt(nl), colt(nl);  // row pass (gathers y), column pass (gathers lambda)
  for (int l = 0; l < nl; ++l) {
    rowt[l].init(m, rsteps, level_group[l], level_group[l]);
    colt[l].init(n, csteps, level_group[l], level_group[l]);
    for (int r = 0; r < m; ++r)
      for (int k = 0; k < rlen(r); ++k)
        ++rowt[l].at(rowt[l].cell(rpos[r], k), rowt[l].cls(cpos[r_col[r_ptr[r] + k]]));
    for (int c = 0; c < n; ++c)
      for (int j = 0; j < clen(c); ++j)
        ++colt[l].at(colt[l].cell(cpos[c], j), colt[l].cls(rpos[c_row[c_ptr[c] + j]]));
  }
  auto total = [&]() {
    int64_t t = 0;
    for (int l = 0; l < nl; ++l) t += rowt[l].total() + colt[l].total();
    return t;
  };
  stats.passes_before = total();

  // Length classes: lines that may trade positions.
  std::vector<std::vector<int>> rclass(rsteps + 1), cclass(csteps + 1);
  for (int r = 0; r < m; ++r) rclass[rlen(r)].push_back(r);
  for (int c = 0; c < n; ++c) cclass[clen(c)].push_back(c);

  std::mt19937_64 rng(0x5EED5u);
  std::vector<Change> changes;
  std::vector<std::pair<Table*, int>> touched;
  uint32_t move_id = 0;
  auto touch = [&](Table& t, int cell) {
    if (t.stamp[cell] != move_id) {
      t.stamp[cell] = move_id;
      touched.push_back({&t, cell});
    }
  };
  auto change = [&](Table& t, int cell, int cls, int delta) {
    t.at(cell, cls) = (uint8_t)(t.at(cell, cls) + delta);
    changes.push_back({&t, cell, cls, delta});
  };

  // One side of the search: lines A (moved) whose own pass gathers the other
  // side's positions (own_t, entries a_ptr/a_idx), and whose positions are
  // gathered by the other side's pass (other_t, entries ent_ptr/ent_line/ent_step).
  auto try_move = [&](bool rows_side) -> bool {
    const int count = rows_side ? m : n;
    std::vector<int>& pos = rows_side ? rpos : cpos;
    const std::vector<int>& opos = rows_side ? cpos : rpos;
    const std::vector<int32_t>& a_ptr = rows_side ? r_ptr : c_ptr;
    const std::vector<int32_t>& a_idx = rows_side ? r_col : c_row;
    const std::vector<int32_t>& e_ptr = rows_side ? rent_ptr : cent_ptr;
    const std::vector<int32_t>& e_line = rows_side ? rent_c : cent_r;
    const std::vector<int32_t>& e_step = rows_side ? rent_j : cent_k;
    std::vector<Table>& own = rows_side ? rowt : colt;
    std::vector<Table>& other = rows_side ? colt : rowt;
    std::vector<std::vector<int>>& cls_lists = rows_side ? rclass : cclass;

    const int x = (int)(rng() % (uint64_t)count);
    const int len = a_ptr[x + 1] - a_ptr[x];
    const std::vector<int>& peers = cls_lists[len];
    const int y = peers[rng() % peers.size()];
    if (x == y) return false;
    const int px = pos[x], py = pos[y];
    // Only lines that take part in a conflict are worth moving.
    bool conflicted = false;
    for (int l = 0; l < nl && !conflicted; ++l) {
      for (int k = 0; k < len && !conflicted; ++k)
        conflicted = own[l].at(own[l].cell(px, k), own[l].cls(opos[a_idx[a_ptr[x] + k]])) > 1;
      for (int e = e_ptr[x]; e < e_ptr[x + 1] && !conflicted; ++e)
        conflicted = other[l].at(other[l].cell(opos[e_line[e]], e_step[e]), other[l].cls(px)) > 1;
    }
    if (!conflicted) return false;
    ++move_id;
    if (move_id == 0) {  // stamp wrap-around
      for (int l = 0; l < nl; ++l) {
        std::fill(rowt[l].stamp.begin(), rowt[l].stamp.end(), 0u);
        std::fill(colt[l].stamp.begin(), colt[l].stamp.end(), 0u);
      }
      move_id = 1;
    }
    touched.clear();
    changes.clear();
    for (int l = 0; l < nl; ++l) {
      Table& ot = own[l];
      Table& tt = other[l];
      if (ot.cell(px, 0) != ot.cell(py, 0)) {
        for (int k = 0; k < len; ++k) {
          const int cx = ot.cell(px, k), cy = ot.cell(py, k);
          touch(ot, cx);
          touch(ot, cy);
        }
      }
      if (tt.cls(px) != tt.cls(py)) {
        for (int e = e_ptr[x]; e < e_ptr[x + 1]; ++e) touch(tt, tt.cell(opos[e_line[e]], e_step[e]));
        for (int e = e_ptr[y]; e < e_ptr[y + 1]; ++e) touch(tt, tt.cell(opos[e_line[e]], e_step[e]));
      }
    }
    if (touched.empty()) return false;
    int64_t before = 0;
    for (auto& t : touched) before += t.first->passes(t.second);
    for (int l = 0; l < nl; ++l) {
      Table& ot = own[l];
      Table& tt = other[l];
      if (ot.cell(px, 0) != ot.cell(py, 0)) {
        for (int k = 0; k < len; ++k) {
          const int cx = ot.cell(px, k), cy = ot.cell(py, k);
          const int bx = ot.cls(opos[a_idx[a_ptr[x] + k]]), by = ot.cls(opos[a_idx[a_ptr[y] + k]]);
          change(ot, cx, bx, -1);
          change(ot, cy, bx, +1);
          change(ot, cy, by, -1);
          change(ot, cx, by, +1);
        }
      }
      if (tt.cls(px) != tt.cls(py)) {
        for (int e = e_ptr[x]; e < e_ptr[x + 1]; ++e) {
          const int c = tt.cell(opos[e_line[e]], e_step[e]);
          change(tt, c, tt.cls(px), -1);
          change(tt, c, tt.cls(py), +1);
        }
        for (int e = e_ptr[y]; e < e_ptr[y + 1]; ++e) {
          const int c = tt.cell(opos[e_line[e]], e_step[e]);
          change(tt, c, tt.cls(py), -1);
          change(tt, c, tt.cls(px), +1);
        }
      }
    }
    int64_t after = 0;
    for (auto& t : touched) after += t.first->passes(t.second);
    if (after <= before) {
      pos[x] = py;
      pos[y] = px;
      return true;
    }
    for (auto it = changes.rbegin(); it != changes.rend(); ++it)
      it->t->at(it->cell, it->cls) = (uint8_t)(it->t->at(it->cell, it->cls) - it->delta);
    return false;
  };

  for (int64_t mv = 0; mv < max_moves; ++mv) {
    const bool rows_side = (rng() % (uint64_t)(m + n)) < (uint64_t)m;
    if (try_move(rows_side)) ++stats.accepted;
  }
  stats.moves = max_moves;
  stats.passes_after = total();
  for (int r = 0; r < m; ++r) row_order[rpos[r]] = r;
  for (int c = 0; c < n; ++c) col_order[cpos[c]] = c;
  return stats;
}

}  // namespace purin
