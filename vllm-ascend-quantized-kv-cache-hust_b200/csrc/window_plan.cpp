// Host planner of the KIVI residual windows (native C++ behind the C-ABI).
//
// Semantics are the reference's residual state machine
// (methods/kivi_int4/attention_backend.py:181-462, :813-836): one ring row of
// `capacity` lanes per live request and side;
//   keys:   a new slot arriving at a full window first flushes the WHOLE
//           window (a whole-group, block-aligned pack into the int4 history,
//           gated by is_aligned_key_window, semantics.py:254-283);
//   values: a new slot arriving at a full window evicts the ONE oldest lane;
//   a slot the window already holds is overwritten in place;
//   prune drops lanes whose slot the request no longer owns and compacts the
//   survivors to lanes 0.. in FIFO order (_set_kivi_residual_window).
//
// The ring state (slot ids, FIFO start and length per row and side) lives in
// caller-owned int64 arrays; the planner keeps pointers to them. A plan
// records, without touching device data, where every new token goes and which
// lanes each flush reads — a lane's content at plan start, or a token written
// earlier in the same plan — so the device applies a whole forward with one
// gather, one pack launch per side and one scatter.
//
// Source codes: s >= 0 is ring lane s (row * capacity + lane), s < 0 is new
// token -1 - s.
#include <algorithm>
#include <cstdint>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "qkv_sm100.h"

#include "window_plan.h"

namespace {

using qkv::win::Side;
using qkv::win::SidePlan;
using qkv::win::Window;

inline int64_t new_src(int64_t t) { return -1 - t; }

// is_aligned_key_window (methods/kivi_int4/semantics.py:254-283): whole
// groups, each contiguous, starting at a group-aligned block offset and
// staying inside one block.
bool aligned_key_window(const int64_t* s, int64_t n, int group, int block_size) {
  if (n == 0 || n % group) return false;
  for (int64_t g0 = 0; g0 < n; g0 += group) {
    const int64_t first = s[g0];
    if ((first % block_size) % group) return false;
    if (s[g0 + group - 1] / block_size != first / block_size) return false;
    for (int i = 1; i < group; ++i)
      if (s[g0 + i] != first + i) return false;
  }
  return true;
}

// lanes of `row` in FIFO order
void fifo_lanes(const Window& w, const Side& sd, int row, std::vector<int>& out) {
  out.clear();
  const int64_t n = sd.length[row];
  const int64_t s = sd.start[row];
  for (int64_t i = 0; i < n; ++i) out.push_back(static_cast<int>((s + i) % w.cap));
}

bool valid(const Window* w, int row) { return w != nullptr && row >= 0 && row < w->rows; }

}  // namespace

extern "C" {

QKV_API void* qkv_window_create(int rows, int capacity, int group_size, int64_t* key_slots, int64_t* key_start,
                                int64_t* key_length, int64_t* value_slots, int64_t* value_start,
                                int64_t* value_length) {
  if (rows <= 0 || capacity <= 0 || group_size <= 0 || !key_slots || !key_start || !key_length || !value_slots ||
      !value_start || !value_length)
    return nullptr;
  Window* w = new (std::nothrow) Window();
  if (w == nullptr) return nullptr;
  w->rows = rows;
  w->cap = capacity;
  w->group = group_size;
  w->side[0] = Side{key_slots, key_start, key_length};
  w->side[1] = Side{value_slots, value_start, value_length};
  for (SidePlan& p : w->plan) p.resize(static_cast<int64_t>(rows) * capacity);
  return w;
}

QKV_API void qkv_window_destroy(void* h) { delete static_cast<Window*>(h); }

QKV_API void qkv_window_begin(void* h) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr) return;
  w->plan[0].clear();
  w->plan[1].clear();
}

QKV_API int qkv_window_store(void* h, int row, int n, const int64_t* slots, const int64_t* tokens, int is_key,
                             int gate_block_size) {
  Window* w = static_cast<Window*>(h);
  if (!valid(w, row) || n < 0 || (n > 0 && (!slots || !tokens))) return QKV_ERR_INVALID;
  const int k = is_key ? 0 : 1;
  Side& sd = w->side[k];
  SidePlan& p = w->plan[k];
  const int cap = w->cap;
  int64_t* rs = sd.slots + static_cast<int64_t>(row) * cap;
  const int64_t base = static_cast<int64_t>(row) * cap;
  std::vector<int64_t>& ev = w->scratch;
  for (int i = 0; i < n; ++i) {
    const int64_t slot = slots[i];
    const int64_t t = tokens[i];
    // a slot the window holds is overwritten in place (first hit in FIFO
    // order: lanes start .. cap - 1, then 0 .. the wrapped end)
    int hit = -1;
    {
      const int64_t st = sd.start[row], len = sd.length[row];
      const int64_t end1 = std::min<int64_t>(st + len, cap);
      for (int64_t l = st; l < end1 && hit < 0; ++l)
        if (rs[l] == slot) hit = static_cast<int>(l);
      for (int64_t l = 0; l < st + len - cap && hit < 0; ++l)
        if (rs[l] == slot) hit = static_cast<int>(l);
    }
    if (hit >= 0) {
      p.set(base + hit, new_src(t));
      continue;
    }
    while (sd.length[row] >= cap) {
      const int count = is_key ? cap : 1;
      const int64_t st = sd.start[row];
      ev.clear();
      for (int j = 0; j < count; ++j) ev.push_back(rs[(st + j) % cap]);
      if (is_key && gate_block_size > 0 &&
          !aligned_key_window(ev.data(), static_cast<int64_t>(ev.size()), w->group, gate_block_size))
        return QKV_ERR_INVALID;
      for (int j = 0; j < count; ++j) {
        const int64_t lane = (st + j) % cap;
        p.flush_src.push_back(p.src_of(base + lane));
        p.flush_slots.push_back(ev[j]);
        rs[lane] = -1;
      }
      p.keep_valid = false;
      sd.length[row] -= count;
      sd.start[row] = sd.length[row] == 0 ? 0 : (st + count) % cap;
    }
    const int64_t tail = (sd.start[row] + sd.length[row]) % cap;
    rs[tail] = slot;
    sd.length[row] += 1;
    p.set(base + tail, new_src(t));
  }
  return QKV_OK;
}

QKV_API int qkv_window_store_one_each(void* h, int n, const int64_t* rows, const int64_t* slots,
                                      const int64_t* tokens, int is_key, int gate_block_size) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr || n < 0 || (n > 0 && (!rows || !slots || !tokens))) return QKV_ERR_INVALID;
  for (int i = 0; i < n; ++i) {
    const int rc = qkv_window_store(h, static_cast<int>(rows[i]), 1, slots + i, tokens + i, is_key,
                                    gate_block_size);
    if (rc != QKV_OK) return rc;
  }
  return QKV_OK;
}

QKV_API int qkv_window_flush_direct(void* h, int n, const int64_t* slots, const int64_t* tokens, int is_key) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr || n < 0 || (n > 0 && (!slots || !tokens))) return QKV_ERR_INVALID;
  SidePlan& p = w->plan[is_key ? 0 : 1];
  for (int i = 0; i < n; ++i) {
    p.flush_src.push_back(new_src(tokens[i]));
    p.flush_slots.push_back(slots[i]);
  }
  p.keep_valid = false;
  return QKV_OK;
}

QKV_API int qkv_window_prune(void* h, int row, int n_live, const int64_t* live_slots, int is_key) {
  Window* w = static_cast<Window*>(h);
  if (!valid(w, row) || n_live < 0 || (n_live > 0 && !live_slots)) return QKV_ERR_INVALID;
  const int k = is_key ? 0 : 1;
  Side& sd = w->side[k];
  SidePlan& p = w->plan[k];
  const int cap = w->cap;
  int64_t* rs = sd.slots + static_cast<int64_t>(row) * cap;
  const int64_t base = static_cast<int64_t>(row) * cap;
  std::vector<int> lanes;
  fifo_lanes(*w, sd, row, lanes);
  if (lanes.empty()) return QKV_OK;
  std::unordered_set<int64_t> live(live_slots, live_slots + n_live);
  std::vector<int64_t> kept_slots, srcs;
  for (int l : lanes)
    if (live.count(rs[l])) {
      kept_slots.push_back(rs[l]);
      srcs.push_back(p.src_of(base + l));
    }
  if (kept_slots.size() == lanes.size()) return QKV_OK;
  std::fill(rs, rs + cap, int64_t{-1});
  std::copy(kept_slots.begin(), kept_slots.end(), rs);
  sd.start[row] = 0;
  sd.length[row] = static_cast<int64_t>(kept_slots.size());
  // the compaction reads the kept lanes' sources (captured above) before
  // anything of this plan lands; it replaces every pending write of the row
  for (int l = 0; l < cap; ++l) p.erase(base + l);
  for (size_t i = 0; i < srcs.size(); ++i) p.set(base + static_cast<int64_t>(i), srcs[i]);
  p.keep_valid = false;
  return QKV_OK;
}

QKV_API int qkv_window_reset_row(void* h, int row) {
  Window* w = static_cast<Window*>(h);
  if (!valid(w, row)) return QKV_ERR_INVALID;
  for (Side& sd : w->side) {
    std::fill(sd.slots + static_cast<int64_t>(row) * w->cap, sd.slots + static_cast<int64_t>(row + 1) * w->cap,
              int64_t{-1});
    sd.start[row] = 0;
    sd.length[row] = 0;
  }
  return QKV_OK;
}

// Deduplicated flush list sizes and the ring writes of the open plan. A
// batched pack has no write order where the reference's sequential flushes
// do, so only the last flush of a slot (keys: of a whole group, found by its
// first slot) is kept. Cached until the plan changes.
static const std::vector<int64_t>& dedupe(Window& w, int is_key) {
  SidePlan& p = w.plan[is_key ? 0 : 1];
  if (p.keep_valid) return p.keep;
  std::vector<int64_t>& keep = p.keep;
  keep.clear();
  const int64_t n = static_cast<int64_t>(p.flush_slots.size());
  if (is_key) {
    const int g = w.group;
    std::unordered_set<int64_t> seen;
    std::vector<int64_t> groups;
    for (int64_t gi = n / g - 1; gi >= 0; --gi)
      if (seen.insert(p.flush_slots[gi * g]).second) groups.push_back(gi);
    std::reverse(groups.begin(), groups.end());
    for (int64_t gi : groups)
      for (int j = 0; j < g; ++j) keep.push_back(gi * g + j);
  } else {
    // the common case (every evicted slot distinct) keeps everything
    std::vector<int64_t>& sorted = w.scratch;
    sorted.assign(p.flush_slots.begin(), p.flush_slots.end());
    std::sort(sorted.begin(), sorted.end());
    if (std::adjacent_find(sorted.begin(), sorted.end()) == sorted.end()) {
      for (int64_t i = 0; i < n; ++i) keep.push_back(i);
    } else {
      std::unordered_map<int64_t, int64_t> last;
      for (int64_t i = 0; i < n; ++i) last[p.flush_slots[i]] = i;
      for (auto& kv : last) keep.push_back(kv.second);
      std::sort(keep.begin(), keep.end());
    }
  }
  p.keep_valid = true;
  return keep;
}

// lanes with a pending write, ascending
static void live_writes(SidePlan& p, std::vector<int64_t>& out) {
  out.clear();
  for (int64_t l : p.touched)
    if (p.write_gen[l] == p.gen) out.push_back(l);
  std::sort(out.begin(), out.end());
}

QKV_API int qkv_window_plan_counts(void* h, int is_key, int64_t* n_flush, int64_t* n_writes) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr || !n_flush || !n_writes) return QKV_ERR_INVALID;
  *n_flush = static_cast<int64_t>(dedupe(*w, is_key).size());
  SidePlan& p = w->plan[is_key ? 0 : 1];
  int64_t nw = 0;
  for (int64_t l : p.touched) nw += p.write_gen[l] == p.gen;
  *n_writes = nw;
  return QKV_OK;
}

QKV_API int qkv_window_plan_export(void* h, int is_key, int64_t* flush_src, int64_t* flush_slots,
                                   int64_t* write_lanes, int64_t* write_src) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr) return QKV_ERR_INVALID;
  const std::vector<int64_t>& keep = dedupe(*w, is_key);
  SidePlan& p = w->plan[is_key ? 0 : 1];
  std::vector<int64_t> lanes;
  live_writes(p, lanes);
  if (!keep.empty() && (!flush_src || !flush_slots)) return QKV_ERR_INVALID;
  if (!lanes.empty() && (!write_lanes || !write_src)) return QKV_ERR_INVALID;
  for (size_t i = 0; i < keep.size(); ++i) {
    flush_src[i] = p.flush_src[keep[i]];
    flush_slots[i] = p.flush_slots[keep[i]];
  }
  for (size_t i = 0; i < lanes.size(); ++i) {
    write_lanes[i] = lanes[i];
    write_src[i] = p.write_val[lanes[i]];
  }
  return QKV_OK;
}

// expected_live for many rows: both windows hold exactly the request's last
// positions (entry i of a window of n slots is position seq_len - n + i).
// table: int64 block-table rows [n, table_cols] (row i for rows[i]).
QKV_API int qkv_window_expected_live(void* h, int n, const int64_t* rows, const int64_t* seq_lens,
                                     const int64_t* table, int table_cols, int block_size, uint8_t* ok) {
  Window* w = static_cast<Window*>(h);
  if (w == nullptr || n < 0 || block_size <= 0 || table_cols <= 0 || (n > 0 && (!rows || !seq_lens || !table || !ok)))
    return QKV_ERR_INVALID;
  for (int i = 0; i < n; ++i) {
    const int64_t row = rows[i], L = seq_lens[i];
    bool good = row >= 0 && row < w->rows;
    for (int k = 0; k < 2 && good; ++k) {
      const Side& sd = w->side[k];
      const int64_t len = sd.length[row];
      if (len > L) {
        good = false;
        break;
      }
      for (int64_t j = 0; j < len; ++j) {
        const int64_t pos = std::max<int64_t>(L - len + j, 0);
        const int64_t col = pos / block_size;
        if (col >= table_cols) {
          good = false;
          break;
        }
        const int64_t blk = table[static_cast<int64_t>(i) * table_cols + col];
        const int64_t got = sd.slots[row * w->cap + (sd.start[row] + j) % w->cap];
        if (blk < 0 || blk * block_size + pos % block_size != got) {
          good = false;
          break;
        }
      }
    }
    ok[i] = good ? 1 : 0;
  }
  return QKV_OK;
}

}  // extern "C"
