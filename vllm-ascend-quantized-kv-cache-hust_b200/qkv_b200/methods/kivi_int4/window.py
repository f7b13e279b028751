"""Host bookkeeping of the KIVI residual windows, planned per forward.

Semantics are the reference's residual state machine
(methods/kivi_int4/attention_backend.py:181-462, :813-836): one ring row of
``residual_length`` lanes per live request and side;

* keys: a new slot arriving at a full window first flushes the WHOLE window
  (a whole-group, block-aligned pack into the int4 history);
* values: a new slot arriving at a full window evicts the ONE oldest lane;
* a slot already held by the window is overwritten in place;
* ``sync`` drops lanes whose slot the request no longer owns and compacts the
  survivors to lanes 0.. in FIFO order.

What differs is execution. The reference walks tokens in Python and launches a
pack per flush, reading slot ids back from the device. Here the slot ids live
in host memory; a ``WindowPlan`` records, without touching device data, where
every token goes and which lanes each flush reads — the lane's content at plan
start, or a token written earlier in the same plan. ``execute`` then does one
gather of the flush inputs, one pack launch per side and one scatter of the
new tokens into the ring, so a decode step costs a constant number of
launches whatever the batch size.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def is_aligned_key_window(slots, group_size: int, block_size: int) -> bool:
    """Whole-group flush gate (the reference's ``is_aligned_key_window``,
    methods/kivi_int4/semantics.py:254-283): every group is contiguous, starts
    at a group-aligned block offset and stays inside one block."""
    n = len(slots)
    if n == 0 or n % group_size:
        return False
    s = np.asarray(slots, dtype=np.int64).reshape(-1, group_size)
    first = s[:, :1]
    if np.any(first % block_size % group_size):
        return False
    if np.any(s[:, -1:] // block_size != first // block_size):
        return False
    return bool(np.all(s == first + np.arange(group_size)))


def ordered_slots(block_table: np.ndarray, seq_lens, block_size: int) -> list[list[int]]:
    """Absolute slot of every live position of each request (the reference's
    ``ordered_slots``, semantics.py:224-252); unallocated (-1) blocks give
    negative slots and are dropped."""
    out = []
    bt = np.asarray(block_table, dtype=np.int64)
    for b, L in enumerate(seq_lens):
        L = int(L)
        if L <= 0:
            out.append([])
            continue
        pos = np.arange(L)
        s = bt[b, pos // block_size] * block_size + pos % block_size
        out.append(s[s >= 0].tolist())
    return out


class RingSide:
    """Slot ids and FIFO state of one side (keys or values) of every row."""

    def __init__(self, rows: int, capacity: int) -> None:
        self.capacity = capacity
        self.slots = np.full((rows, capacity), -1, dtype=np.int64)
        self.start = np.zeros(rows, dtype=np.int64)
        self.length = np.zeros(rows, dtype=np.int64)

    def lanes(self, row: int) -> list[int]:
        n = int(self.length[row])
        if n <= 0:
            return []
        s, cap = int(self.start[row]), self.capacity
        end = s + n
        if end <= cap:
            return list(range(s, end))
        return list(range(s, cap)) + list(range(0, end % cap))

    def reset(self, row: int) -> None:
        self.slots[row].fill(-1)
        self.start[row] = 0
        self.length[row] = 0


# A flush/scatter source: ("ring", flat lane index) or ("new", token index).
Source = tuple


@dataclass
class SidePlan:
    """Pending work of one side for one forward."""

    flush_src: list = field(default_factory=list)    # Source per flushed token
    flush_slots: list = field(default_factory=list)  # its slot
    ring_writes: dict = field(default_factory=dict)  # flat lane -> Source
    compactions: list = field(default_factory=list)  # (row, [old lanes in FIFO order])

    def empty(self) -> bool:
        return not (self.flush_src or self.ring_writes or self.compactions)


class WindowPlanner:
    """Plans residual-window updates for both sides on the host mirror."""

    def __init__(self, rows: int, capacity: int, group_size: int) -> None:
        self.rows = rows
        self.capacity = capacity
        self.group_size = group_size
        self.key = RingSide(rows, capacity)
        self.value = RingSide(rows, capacity)
        # lane -> Source of its current content within the open plan
        self._lane_src: dict[tuple[bool, int], Source] = {}

    def side(self, is_key: bool) -> RingSide:
        return self.key if is_key else self.value

    def begin(self) -> tuple[SidePlan, SidePlan]:
        self._lane_src = {}
        return SidePlan(), SidePlan()

    def _src_of(self, is_key: bool, flat: int) -> Source:
        return self._lane_src.get((is_key, flat), ("ring", flat))

    def store(self, plan: SidePlan, row: int, slots, token_index, *, is_key: bool,
              on_flush=None) -> None:
        """Appends tokens (``slots[i]`` holding new token ``token_index[i]``) to
        ``row``; records flushes and the final lane contents in ``plan``.
        ``on_flush(slots)`` may veto a key flush by raising (alignment gate)."""
        side = self.side(is_key)
        cap = self.capacity
        rs = side.slots[row]
        if len(slots) <= 4:  # decode-sized: search the row instead of indexing it
            lane_of = {}
            for slot in slots:
                hit = np.flatnonzero(rs == int(slot))
                if hit.size:
                    lane_of[int(slot)] = int(hit[0])
        else:
            lane_of = {int(s): lane for lane, s in enumerate(rs.tolist()) if s >= 0}
        base = row * cap
        for slot, t in zip(slots, token_index):
            slot = int(slot)
            lane = lane_of.get(slot)
            if lane is not None:
                self._lane_src[(is_key, base + lane)] = ("new", int(t))
                plan.ring_writes[base + lane] = ("new", int(t))
                continue
            while side.length[row] >= cap:
                count = cap if is_key else 1
                evicted = side.lanes(row)[:count]
                ev_slots = [int(rs[l]) for l in evicted]
                if on_flush is not None:
                    on_flush(ev_slots)
                for l, s in zip(evicted, ev_slots):
                    plan.flush_src.append(self._src_of(is_key, base + l))
                    plan.flush_slots.append(s)
                    lane_of.pop(s, None)
                    rs[l] = -1
                side.length[row] -= count
                side.start[row] = 0 if side.length[row] == 0 else (side.start[row] + count) % cap
            tail = (side.start[row] + side.length[row]) % cap
            rs[tail] = slot
            side.length[row] += 1
            lane_of[slot] = tail
            self._lane_src[(is_key, base + tail)] = ("new", int(t))
            plan.ring_writes[base + tail] = ("new", int(t))

    def store_one_each(self, plan: SidePlan, rows, slots, token_index, *, is_key: bool,
                       on_flush=None) -> None:
        """``store`` of one token per row for a batch of distinct rows (a
        decode step), vectorised: in-place hits, appends and one-lane value
        evictions are array operations; a key window that must flush (a full
        row) takes the per-row path with its alignment gate."""
        rows = np.asarray(rows, dtype=np.int64)
        slots = np.asarray(slots, dtype=np.int64)
        tokens = np.asarray(token_index, dtype=np.int64)
        if rows.size == 0:
            return
        side = self.side(is_key)
        cap = self.capacity
        rs = side.slots[rows]                            # [n, cap] (copy)
        eq = rs == slots[:, None]
        hit = eq.any(axis=1)
        full = side.length[rows] >= cap
        slow = ~hit & full if is_key else np.zeros_like(hit)
        for i in np.flatnonzero(slow):                   # whole-window key flush
            self.store(plan, int(rows[i]), [int(slots[i])], [int(tokens[i])], is_key=True, on_flush=on_flush)
        fast = ~slow
        # in-place overwrites
        hit_lane = eq.argmax(axis=1)
        # value windows at capacity drop their oldest lane first
        ev = fast & ~hit & full
        if ev.any():
            er = rows[ev]
            ev_lane = side.start[er] % cap
            ev_slot = side.slots[er, ev_lane]
            for r, l, sl in zip(er.tolist(), ev_lane.tolist(), ev_slot.tolist()):
                plan.flush_src.append(self._src_of(is_key, r * cap + l))
                plan.flush_slots.append(int(sl))
            side.slots[er, ev_lane] = -1
            side.length[er] -= 1
            side.start[er] = np.where(side.length[er] == 0, 0, (side.start[er] + 1) % cap)
        app = fast & ~hit
        ar = rows[app]
        tail = (side.start[ar] + side.length[ar]) % cap
        side.slots[ar, tail] = slots[app]
        side.length[ar] += 1
        lane = np.where(hit, hit_lane, 0)
        lane[app] = tail
        for r, l, t in zip(rows[fast].tolist(), lane[fast].tolist(), tokens[fast].tolist()):
            flat = r * cap + l
            self._lane_src[(is_key, flat)] = ("new", t)
            plan.ring_writes[flat] = ("new", t)

    def flush_direct(self, plan: SidePlan, slots, token_index) -> None:
        """Records tokens that go straight to the int4 history (bulk prefill)."""
        for slot, t in zip(slots, token_index):
            plan.flush_src.append(("new", int(t)))
            plan.flush_slots.append(int(slot))

    def prune(self, plan: SidePlan, row: int, live: set, *, is_key: bool) -> None:
        """Drops lanes whose slot is not in ``live``; survivors move to lanes
        0.. in FIFO order (the reference's ``_set_kivi_residual_window``)."""
        side = self.side(is_key)
        lanes = side.lanes(row)
        if not lanes:
            return
        rs = side.slots[row]
        keep = [l for l in lanes if int(rs[l]) in live]
        if len(keep) == len(lanes):
            return
        kept_slots = [int(rs[l]) for l in keep]
        base = row * self.capacity
        srcs = [self._src_of(is_key, base + l) for l in keep]
        rs.fill(-1)
        rs[: len(keep)] = kept_slots
        side.start[row] = 0
        side.length[row] = len(keep)
        # the compaction reads the kept lanes' sources (captured above) before
        # anything of this plan lands; it replaces every pending write of the row
        for l in range(self.capacity):
            plan.ring_writes.pop(base + l, None)
            self._lane_src.pop((is_key, base + l), None)
        for new_lane, src in enumerate(srcs):
            plan.ring_writes[base + new_lane] = src
            self._lane_src[(is_key, base + new_lane)] = src

    def window(self, row: int, *, is_key: bool) -> tuple[list[int], list[int]]:
        """(slots in FIFO order, lanes) of a row."""
        side = self.side(is_key)
        lanes = side.lanes(row)
        return [int(side.slots[row, l]) for l in lanes], lanes

    def expected_live_rows(self, rows, seq_lens, table: np.ndarray, block_size: int) -> np.ndarray:
        """``expected_live`` for many rows at once; ``table[i]`` is the block
        table row of ``rows[i]``'s request."""
        rows = np.asarray(rows, dtype=np.int64)
        L = np.asarray(seq_lens, dtype=np.int64)
        ok = np.ones(rows.size, dtype=bool)
        if rows.size == 0:
            return ok
        cap = self.capacity
        ar = np.arange(cap, dtype=np.int64)
        table = np.asarray(table, dtype=np.int64)
        for side in (self.key, self.value):
            n = side.length[rows]
            ok &= n <= L
            valid = ar[None, :] < n[:, None]
            pos = np.clip(L[:, None] - n[:, None] + ar[None, :], 0, None)
            col = np.minimum(pos // block_size, table.shape[1] - 1)
            blocks = np.take_along_axis(table, col, axis=1)
            want = blocks * block_size + pos % block_size
            got = side.slots[rows[:, None], (side.start[rows][:, None] + ar[None, :]) % cap]
            good = (want == got) & (blocks >= 0) & (pos // block_size < table.shape[1])
            ok &= np.all(good | ~valid, axis=1)
        return ok

    def expected_live(self, row: int, seq_len: int, table_row: np.ndarray, block_size: int) -> bool:
        """Fast check that both windows hold exactly the request's last
        positions (the normal case): window entry i of a window of n slots is
        position seq_len - n + i."""
        for side in (self.key, self.value):
            lanes = side.lanes(row)
            n = len(lanes)
            if n == 0:
                continue
            if n > seq_len:
                return False
            pos = np.arange(seq_len - n, seq_len)
            blocks = table_row[pos // block_size].astype(np.int64)
            want = blocks * block_size + pos % block_size
            got = side.slots[row, lanes]
            if np.any(blocks < 0) or not np.array_equal(want, got):
                return False
        return True


__all__ = ["RingSide", "SidePlan", "WindowPlanner", "is_aligned_key_window", "ordered_slots"]
