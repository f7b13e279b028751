// Internal state of the residual-window planner (window_plan.cpp), shared
// with the native decode step (kivi_step.cu). Not part of the C-ABI.
#pragma once

#include <cstdint>
#include <map>
#include <unordered_map>
#include <vector>

namespace qkv {
namespace win {

struct Side {
  int64_t* slots;   // [rows, capacity], -1 = empty lane
  int64_t* start;   // [rows]
  int64_t* length;  // [rows]
};

struct SidePlan {
  std::vector<int64_t> flush_src, flush_slots;
  std::map<int64_t, int64_t> ring_writes;         // flat lane -> source (sorted by lane)
  std::unordered_map<int64_t, int64_t> lane_src;  // flat lane -> source of its content in this plan
  void clear() {
    flush_src.clear();
    flush_slots.clear();
    ring_writes.clear();
    lane_src.clear();
  }
};

struct Window {
  int rows, cap, group;
  Side side[2];  // 0 = key, 1 = value
  SidePlan plan[2];
};

}  // namespace win
}  // namespace qkv
