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
in host memory (numpy arrays shared with the native planner,
``qkv_window_*`` in libqkv_sm100.so); a plan records, without touching device
data, where every token goes and which lanes each flush reads — the lane's
content at plan start, or a token written earlier in the same plan. The mixin
then applies it with one gather, one pack launch per side and one scatter, so
a decode step costs a constant number of launches whatever the batch size.
"""

from __future__ import annotations

import ctypes

import numpy as np

from ...ops import _lib


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


KEY_FLUSH_ERROR = "KIVI key flush requires contiguous aligned token groups."


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _i64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64).reshape(-1))


class SidePlan:
    """Handle on one side (keys or values) of the planner's open plan."""

    def __init__(self, planner: WindowPlanner, is_key: bool) -> None:
        self._planner = planner
        self.is_key = is_key

    def export(self) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        """(flush sources, flush slots, write lanes, write sources), int64.
        Source s >= 0 is ring lane s (row * capacity + lane), s < 0 new token
        -1 - s; only the last flush of a slot (keys: of a whole group) is
        kept, write lanes ascend."""
        lib = _lib.load()
        nf, nw = ctypes.c_int64(0), ctypes.c_int64(0)
        h = self._planner._handle
        _lib.check(lib.qkv_window_plan_counts(h, int(self.is_key), ctypes.byref(nf), ctypes.byref(nw)),
                   "qkv_window_plan_counts")
        out = [np.empty(nf.value, np.int64), np.empty(nf.value, np.int64), np.empty(nw.value, np.int64),
               np.empty(nw.value, np.int64)]
        _lib.check(lib.qkv_window_plan_export(h, int(self.is_key), *(_p(a) for a in out)), "qkv_window_plan_export")
        return tuple(out)

    def empty(self) -> bool:
        f, _, w, _ = self.export()
        return f.size == 0 and w.size == 0


class WindowPlanner:
    """Plans residual-window updates for both sides on the host mirror; the
    state machine runs in the native planner over this object's arrays."""

    def __init__(self, rows: int, capacity: int, group_size: int) -> None:
        self.rows = rows
        self.capacity = capacity
        self.group_size = group_size
        self.key = RingSide(rows, capacity)
        self.value = RingSide(rows, capacity)
        self._lib = _lib.load()
        self._handle = self._lib.qkv_window_create(
            rows, capacity, group_size, _p(self.key.slots), _p(self.key.start), _p(self.key.length),
            _p(self.value.slots), _p(self.value.start), _p(self.value.length))
        if not self._handle:
            raise RuntimeError(f"qkv_window_create failed (rows={rows}, capacity={capacity}, group={group_size})")

    def __del__(self) -> None:
        h, self._handle = getattr(self, "_handle", None), None
        if h:
            self._lib.qkv_window_destroy(h)

    def side(self, is_key: bool) -> RingSide:
        return self.key if is_key else self.value

    def begin(self) -> tuple[SidePlan, SidePlan]:
        self._lib.qkv_window_begin(self._handle)
        return SidePlan(self, True), SidePlan(self, False)

    def _gate_rc(self, rc: int, what: str) -> None:
        if rc == _lib.QKV_ERR_INVALID:
            raise RuntimeError(KEY_FLUSH_ERROR)
        _lib.check(rc, what)

    def store(self, plan: SidePlan, row: int, slots, token_index, *, is_key: bool, gate_block_size: int = 0) -> None:
        """Appends tokens (``slots[i]`` holding new token ``token_index[i]``) to
        ``row``; records flushes and the final lane contents in the open plan.
        A key flush of a window that is not whole aligned groups of
        ``gate_block_size`` blocks raises the reference's RuntimeError."""
        s, t = _i64(slots), _i64(token_index)
        if not 0 <= row < self.rows:
            raise RuntimeError(f"residual row {row} out of range")
        rc = self._lib.qkv_window_store(self._handle, int(row), s.size, _p(s), _p(t), int(is_key),
                                        int(gate_block_size) if is_key else 0)
        self._gate_rc(rc, "qkv_window_store")

    def store_one_each(self, plan: SidePlan, rows, slots, token_index, *, is_key: bool,
                       gate_block_size: int = 0) -> None:
        """``store`` of one token per row for a batch of distinct rows (a
        decode step)."""
        r, s, t = _i64(rows), _i64(slots), _i64(token_index)
        if r.size and (r.min() < 0 or r.max() >= self.rows):
            raise RuntimeError("residual row out of range")
        rc = self._lib.qkv_window_store_one_each(self._handle, r.size, _p(r), _p(s), _p(t), int(is_key),
                                                 int(gate_block_size) if is_key else 0)
        self._gate_rc(rc, "qkv_window_store_one_each")

    def flush_direct(self, plan: SidePlan, slots, token_index) -> None:
        """Records tokens that go straight to the int4 history (bulk prefill)."""
        s, t = _i64(slots), _i64(token_index)
        _lib.check(self._lib.qkv_window_flush_direct(self._handle, s.size, _p(s), _p(t), int(plan.is_key)),
                   "qkv_window_flush_direct")

    def prune(self, plan: SidePlan, row: int, live, *, is_key: bool) -> None:
        """Drops lanes whose slot is not in ``live``; survivors move to lanes
        0.. in FIFO order (the reference's ``_set_kivi_residual_window``)."""
        lv = _i64(sorted(live))
        _lib.check(self._lib.qkv_window_prune(self._handle, int(row), lv.size, _p(lv), int(is_key)),
                   "qkv_window_prune")

    def reset(self, row: int) -> None:
        _lib.check(self._lib.qkv_window_reset_row(self._handle, int(row)), "qkv_window_reset_row")

    def window(self, row: int, *, is_key: bool) -> tuple[list[int], list[int]]:
        """(slots in FIFO order, lanes) of a row."""
        side = self.side(is_key)
        lanes = side.lanes(row)
        return [int(side.slots[row, l]) for l in lanes], lanes

    def expected_live_rows(self, rows, seq_lens, table: np.ndarray, block_size: int) -> np.ndarray:
        """For each ``rows[i]``: both windows hold exactly the last positions of
        a request of ``seq_lens[i]`` tokens (``table[i]`` its block-table
        row); window entry j of a window of n slots is position L - n + j."""
        r, L = _i64(rows), _i64(seq_lens)
        ok = np.ones(r.size, dtype=np.uint8)
        if r.size == 0:
            return ok.astype(bool)
        tb = np.ascontiguousarray(np.asarray(table, dtype=np.int64).reshape(r.size, -1))
        _lib.check(self._lib.qkv_window_expected_live(self._handle, r.size, _p(r), _p(L), _p(tb), tb.shape[1],
                                                      int(block_size), _p(ok)), "qkv_window_expected_live")
        return ok.astype(bool)

    def expected_live(self, row: int, seq_len: int, table_row: np.ndarray, block_size: int) -> bool:
        return bool(self.expected_live_rows([row], [seq_len], np.asarray(table_row)[None, :], block_size)[0])


__all__ = ["KEY_FLUSH_ERROR", "RingSide", "SidePlan", "WindowPlanner", "is_aligned_key_window", "ordered_slots"]
