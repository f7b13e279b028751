// Internal state of the residual-window planner (window_plan.cpp), shared
// with the native decode step (kivi_step.cu). Not part of the C-ABI.
#pragma once

#include <algorithm>
#include <cstdint>
#include <vector>

namespace qkv {
namespace win {

struct Side {
  int64_t* slots;   // [rows, capacity], -1 = empty lane
  int64_t* start;   // [rows]
  int64_t* length;  // [rows]
};

// One side's open plan. Per flat lane (row * capacity + lane) two dense
// entries stamped with the plan's generation, so a new plan clears nothing:
//   src:   where the lane's content comes from in this plan (a token written
//          earlier in it, or a lane it was compacted from), if not itself;
//   write: the pending ring write of the lane, if any.
// `touched` lists the lanes that got a write entry (once each, any order).
struct SidePlan {
  std::vector<int64_t> flush_src, flush_slots;
  std::vector<int64_t> src_val, write_val;
  std::vector<uint32_t> src_gen, write_gen;
  std::vector<int64_t> touched;
  uint32_t gen = 1;
  // flush entries kept after deduplication (cached until the plan changes)
  std::vector<int64_t> keep;
  bool keep_valid = false;

  void resize(int64_t lanes) {
    src_val.assign(lanes, 0);
    write_val.assign(lanes, 0);
    src_gen.assign(lanes, 0);
    write_gen.assign(lanes, 0);
  }
  void clear() {
    flush_src.clear();
    flush_slots.clear();
    touched.clear();
    keep_valid = false;
    if (++gen == 0) {  // generation wrapped: stamps of 0 mean "none"
      std::fill(src_gen.begin(), src_gen.end(), 0u);
      std::fill(write_gen.begin(), write_gen.end(), 0u);
      gen = 1;
    }
  }
  int64_t src_of(int64_t flat) const { return src_gen[flat] == gen ? src_val[flat] : flat; }
  void set(int64_t flat, int64_t src) {
    src_val[flat] = src;
    src_gen[flat] = gen;
    if (write_gen[flat] != gen) touched.push_back(flat);
    write_val[flat] = src;
    write_gen[flat] = gen;
    keep_valid = false;
  }
  void erase(int64_t flat) {
    src_gen[flat] = 0;
    write_gen[flat] = 0;
  }
};

struct Window {
  int rows, cap, group;
  Side side[2];  // 0 = key, 1 = value
  SidePlan plan[2];
  std::vector<int64_t> scratch;  // flush slots of one eviction
};

}  // namespace win
}  // namespace qkv
