"""Restatement of the TOPK-32 capture unit and its AMAX32 scan (TEST ORACLE).

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` as the checker of the CUDA
top-k kernels (``f5_topk32_*``); the product path never imports it.

Follows the numpy model of coreyhahn/fable5_llm's RUNG-4 top-k block,
``tb/scripts/gen_topk_cases.py:75-102`` (``Ref.fresh`` / ``Ref.push``), whose
semantics that file derives from ``rtl/vec_alu.sv``:

* the element counter ``am_g`` is 18 bits wide and wraps (:57-58, :93);
  it restarts only on a "fresh" command (:84-89);
* AMAX32 keeps the first maximum (strictly-greater update, :89-92);
* the list holds at most 32 (value, index) entries sorted by value
  descending, ties by arrival; an arriving element goes after every entry
  with value >= its own (:95-99); a full list rejects an element whose value
  is <= entry[31] (:100-111);
* ``ovf_lit``: a rejected element tied entry[31]; ``ovf_disp``: that, or an
  insertion displaced an element equal to the new entry[31] (:106-111).

Pinned against the fixtures ``tests/golden/topk_cases.npz`` that the
reference's own generator produced (``tests/golden/gen_topk_golden.py``).
"""
from __future__ import annotations

import numpy as np

NENT = 32
IDXW = 18
IDXM = (1 << IDXW) - 1


class TopKUnit:
    """Sequential model: ``push`` one int32 value at a time."""

    def __init__(self, idx_bits: int = IDXW):
        self.mask = (1 << idx_bits) - 1
        self.am_g = 0
        self.am_first = True
        self.am_idx = 0
        self.am_val = 0
        self.fresh()
        self.nelem = 0

    def fresh(self):
        self.am_g = 0
        self.am_first = True
        self.entries = []          # [(value, index)], value descending, stable
        self.ovf_lit = False
        self.ovf_disp = False

    def push(self, v: int):
        idx = self.am_g & self.mask
        if self.am_first or v > self.am_val:
            self.am_val, self.am_idx = v, idx
        self.am_first = False
        self.am_g = (self.am_g + 1) & self.mask
        self.nelem += 1
        lst = self.entries
        if len(lst) == NENT:
            last = lst[-1][0]
            if v < last:
                return
            if v == last:
                self.ovf_lit = self.ovf_disp = True
                return
        # insertion point: after every entry whose value is >= v
        pos = len(lst)
        while pos > 0 and lst[pos - 1][0] < v:
            pos -= 1
        lst.insert(pos, (v, idx))
        if len(lst) > NENT:
            dropped = lst.pop()
            if dropped[0] == lst[-1][0]:
                self.ovf_disp = True

    def result(self) -> dict:
        return {"count": len(self.entries),
                "val": np.array([e[0] for e in self.entries], dtype=np.int64),
                "idx": np.array([e[1] for e in self.entries], dtype=np.int64),
                "ovf_lit": int(self.ovf_lit), "ovf_disp": int(self.ovf_disp),
                "amax_idx": int(self.am_idx), "amax_val": int(self.am_val)}


def topk32(values, idx_bits: int = 31) -> dict:
    """One fresh scan over ``values`` (int32, arrival order).  With the
    default 31-bit counter the index is the element's position."""
    u = TopKUnit(idx_bits)
    for v in np.asarray(values, dtype=np.int64).tolist():
        u.push(int(v))
    return u.result()


def run_commands(elements, cmds, idx_bits: int = IDXW) -> dict:
    """The unit driven by AMAX32 commands ``(element offset, length, fresh)``
    over the element array (the way tb_topk.sv drives it)."""
    u = TopKUnit(idx_bits)
    el = np.asarray(elements, dtype=np.int64)
    for off, ln, fresh in cmds:
        if fresh:
            u.fresh()
        for v in el[off:off + ln].tolist():
            u.push(int(v))
    return u.result()


def flatten_after_fresh(elements, cmds) -> np.ndarray:
    """The element sequence the unit holds at the end: everything pushed
    since the last fresh command, in arrival order."""
    el = np.asarray(elements, dtype=np.int64)
    start = max(i for i, c in enumerate(cmds) if c[2]) if any(c[2] for c in cmds) else 0
    parts = [el[off:off + ln] for off, ln, _ in cmds[start:]]
    return np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
