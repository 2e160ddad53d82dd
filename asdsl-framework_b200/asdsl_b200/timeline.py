"""Per-CTA timeline of the streaming GEMV launches (``asdsl_b200_timeline_set``).

The reference prints a per-stage breakdown of a decode token when ASDSL_ENGINE_PROFILE is set
(asdsl/kernels/native/unified_engine.cpp:74-90, :1675).  The per-op chain here is one kernel per
projection, so its breakdown is a timeline: while a capture is active, every CTA of every
streaming GEMV appends %globaltimer records of its start, the end of its dependency wait, the end
of its activation prologue, the end of its consumers and the producer's last copy.

    with Timeline(device) as tl:
        ...  # launches (eager or graph replays)
    launches = tl.launches()          # one dict per launch instance, in start order
    print(format_chain(launches))
"""

from __future__ import annotations

import ctypes
from collections import defaultdict

import numpy as np

from . import _lib

REC = np.dtype([("code", "<u4"), ("id", "<u4"), ("where", "<u4"), ("pad", "<u4"),
                ("t", "<u8"), ("pad2", "<u8")])
START, WAITED, PROLOGUE, CONSUMED, END, PRODUCED = 1, 2, 3, 4, 5, 6
_EVENTS = {START: "start", WAITED: "waited", PROLOGUE: "prologue", CONSUMED: "consumed", END: "end",
           PRODUCED: "produced"}


class Timeline:
    """Device record buffer of ``capacity`` records, active inside the ``with`` block."""

    def __init__(self, device=None, capacity: int = 1 << 20):
        import torch

        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.capacity = int(capacity)
        self.buf = torch.zeros(self.capacity * REC.itemsize, dtype=torch.uint8, device=self.device)
        self.recs = np.zeros(0, dtype=REC)
        self.dropped = 0

    def __enter__(self):
        _lib.call("asdsl_b200_timeline_set", ctypes.c_void_p(self.buf.data_ptr()), self.capacity)
        return self

    def __exit__(self, *exc):
        n = ctypes.c_uint(0)
        _lib.call("asdsl_b200_timeline_count", ctypes.byref(n))
        _lib.call("asdsl_b200_timeline_set", None, 0)
        kept = min(int(n.value), self.capacity)
        self.dropped = int(n.value) - kept
        self.recs = self.buf[: kept * REC.itemsize].cpu().numpy().view(REC).copy()
        return False

    def launches(self) -> list[dict]:
        return group_launches(self.recs)


def kernel_name(code: int) -> str:
    fmt, pro, epi, nt = (code >> 4) & 15, (code >> 8) & 15, (code >> 12) & 15, (code >> 16) & 255
    return f"k_stream_gemv<{fmt},{pro},{epi},{nt}>"


def group_launches(recs: np.ndarray) -> list[dict]:
    """Records -> launch instances.  A graph replays its launches under the launch numbers given
    at capture, so the k-th record of (launch number, block, event) belongs to the k-th instance
    of that launch number."""
    occ: dict = defaultdict(int)
    inst: dict = defaultdict(lambda: defaultdict(list))
    names: dict = {}
    for r in recs[np.argsort(recs["t"], kind="stable")]:
        ev = int(r["code"]) & 15
        lid, blk = int(r["id"]), int(r["where"]) & 0xFFFFF
        k = occ[(lid, blk, ev)]
        occ[(lid, blk, ev)] = k + 1
        inst[(lid, k)][ev].append(int(r["t"]))
        names[lid] = kernel_name(int(r["code"]))
    out = []
    for (lid, k), evs in inst.items():
        if START not in evs or END not in evs:
            continue
        d = {"id": lid, "instance": k, "kernel": names[lid], "ctas": len(evs[START])}
        for ev, nm in _EVENTS.items():
            if ev in evs:
                d[nm + "_min"] = min(evs[ev])
                d[nm + "_max"] = max(evs[ev])
        out.append(d)
    out.sort(key=lambda d: d["start_min"])
    return out


def chain_rows(launches: list[dict]) -> list[dict]:
    """Per launch, in microseconds: its span (first CTA start to last CTA end), the spread of
    CTA starts, how long after the previous launch's last CTA ended its consumers got past the
    dependency wait, the prologue (last wait -> last prologue end), the consumers' spread of
    ends, and the producer's last copy relative to the last end."""
    rows = []
    prev = None
    for d in launches:
        us = lambda a, b: (d[a] - d[b]) / 1e3  # noqa: E731
        row = {
            "kernel": d["kernel"], "id": d["id"], "ctas": d["ctas"],
            "span": us("end_max", "start_min"),
            "start_spread": us("start_max", "start_min"),
            "prologue": us("prologue_max", "waited_max") if "prologue_max" in d else None,
            "end_spread": us("end_max", "end_min"),
            "produced_before_end": us("end_max", "produced_max") if "produced_max" in d else None,
        }
        if prev is not None:
            row["start_after_prev_end"] = (d["start_min"] - prev["end_max"]) / 1e3
            row["waited_after_prev_end"] = (d["waited_min"] - prev["end_max"]) / 1e3
            row["end_after_prev_end"] = (d["end_max"] - prev["end_max"]) / 1e3
        rows.append(row)
        prev = d
    return rows


def summarize(rows: list[dict], period: int | None = None) -> dict:
    """Mean of every figure per kernel template (the first launch of a chain has no predecessor).
    With ``period``, launches are also told apart by their place in a repeating pattern of launch
    numbers (the graph of one decode step: period 4 = qkv, o, gate_up, down)."""
    acc: dict = defaultdict(lambda: defaultdict(list))
    id0 = min((r["id"] for r in rows), default=0)
    for r in rows:
        key = r["kernel"] if period is None else f"{r['kernel']} [{(r['id'] - id0) % period}]"
        for k, v in r.items():
            if isinstance(v, float):
                acc[key][k].append(v)
    return {kern: {k: round(float(np.mean(v)), 3) for k, v in figs.items()} | {"launches": len(figs["span"])}
            for kern, figs in acc.items()}


def format_chain(launches: list[dict], period: int | None = None) -> str:
    rows = chain_rows(launches)
    summ = summarize(rows, period)
    cols = ["launches", "span", "end_after_prev_end", "start_after_prev_end", "waited_after_prev_end", "prologue",
            "start_spread", "end_spread", "produced_before_end"]
    lines = ["kernel                              " + " ".join(f"{c[:14]:>14}" for c in cols)]
    for kern, f in summ.items():
        lines.append(f"{kern:36}" + " ".join(f"{f.get(c, float('nan')):14.3f}" for c in cols))
    return "\n".join(lines)
