"""Per-CTA timeline of the streaming GEMV launches (``asdsl_b200_timeline_set``).

The reference prints a per-stage breakdown of a decode token when ASDSL_ENGINE_PROFILE is set
(asdsl/kernels/native/unified_engine.cpp:74-90, :1675).  The per-op chain here is one kernel per
projection, so its breakdown is a timeline: while a capture is active, every CTA of every
streaming GEMV writes %globaltimer records of its start, the end of its dependency wait, the
arrival of its activation, the RMSNorm reduction, the end of its activation prologue, the end of
its consumers and the producer's last copy.

    with Timeline(device) as tl:
        ...  # launches (eager or graph replays)
    launches = tl.launches()          # one dict per launch instance, in start order
    print(format_chain(launches))

The records are compiled only into libasdsl_b200_timeline.so (the default library's kernels carry
no hooks): set ASDSL_B200_TIMELINE=1 before asdsl_b200 loads its library, or load it explicitly
with ``_lib.load(_lib.TIMELINE_LIB_PATH)``.
"""

from __future__ import annotations

import ctypes
from collections import defaultdict

import numpy as np

from . import _lib

REC = np.dtype([("t", "<u8"), ("code", "<u4"), ("id", "<u4")])
# records as read back: the device record plus its block (from its place in the buffer)
ROW = np.dtype([("t", "<u8"), ("code", "<u4"), ("id", "<u4"), ("block", "<u4")])
REDUCED, START, WAITED, PROLOGUE, CONSUMED, END, PRODUCED, XLOADED, FIRST_FULL, LAST_FULL, XALL = range(11)
# k_attention_exact's phases (its records carry template code 15)
A_ROPE, A_SCORES, A_MAXIMA, A_WEIGHTS, A_SUMS = range(11, 16)
_EVENTS = {START: "start", WAITED: "waited", PROLOGUE: "prologue", CONSUMED: "consumed", END: "end",
           PRODUCED: "produced", XLOADED: "xloaded", REDUCED: "reduced", FIRST_FULL: "first_full",
           LAST_FULL: "last_full", XALL: "xall", A_ROPE: "rope", A_SCORES: "scores", A_MAXIMA: "maxima",
           A_WEIGHTS: "weights", A_SUMS: "sums"}
ATTN_PHASES = ["start", "waited", "rope", "scores", "maxima", "weights", "sums", "end"]
MAX_BLOCKS, EVENTS = 1024, 16


class Timeline:
    """Device record buffer of ``slots`` CTAs per block index, active inside the ``with`` block."""

    def __init__(self, device=None, slots: int = 320):
        import torch

        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.slots = int(slots)
        nbytes = int(_lib.load().asdsl_b200_timeline_bytes(self.slots))
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.recs = np.zeros(0, dtype=ROW)
        self.dropped = 0

    def __enter__(self):
        _lib.call("asdsl_b200_timeline_set", ctypes.c_void_p(self.buf.data_ptr()), self.slots)
        return self

    def __exit__(self, *exc):
        import torch

        torch.cuda.synchronize(self.device)
        _lib.call("asdsl_b200_timeline_set", None, 0)
        raw = self.buf.cpu().numpy()
        cnt = raw[: 4 * MAX_BLOCKS].view("<u4")
        self.dropped = int(np.maximum(cnt.astype(np.int64) - self.slots, 0).sum())
        recs = raw[4 * MAX_BLOCKS:].view(REC).reshape(MAX_BLOCKS, self.slots, EVENTS)
        blk = np.broadcast_to(np.arange(MAX_BLOCKS, dtype=np.uint32)[:, None, None], recs.shape)
        live = recs["t"] != 0
        out = np.zeros(int(live.sum()), dtype=ROW)
        for f in ("t", "code", "id"):
            out[f] = recs[f][live]
        out["block"] = blk[live]
        self.recs = out
        return False

    def launches(self) -> list[dict]:
        return group_launches(self.recs)


def kernel_name(code: int) -> str:
    fmt, pro, epi, nt = (code >> 4) & 15, (code >> 8) & 15, (code >> 12) & 15, (code >> 16) & 255  # SM in bits 24+
    if fmt == 15:
        return "k_attention_exact"
    return f"k_stream_gemv<{fmt},{pro},{epi},{nt}>"


def group_launches(recs: np.ndarray) -> list[dict]:
    """Records -> launch instances.  A graph replays its launches under the launch numbers given
    at capture, so the k-th record of (launch number, block, event) belongs to the k-th instance
    of that launch number.  Each instance keeps the earliest and latest time of every event and
    the per-CTA times (``ctas``: block -> {event name: t})."""
    occ: dict = defaultdict(int)
    inst: dict = defaultdict(lambda: defaultdict(dict))
    names: dict = {}
    for r in recs[np.argsort(recs["t"], kind="stable")]:
        ev = int(r["code"]) & 15
        lid, blk = int(r["id"]), int(r["block"])
        k = occ[(lid, blk, ev)]
        occ[(lid, blk, ev)] = k + 1
        inst[(lid, k)][blk][_EVENTS.get(ev, str(ev))] = int(r["t"])
        names[lid] = kernel_name(int(r["code"]))
    out = []
    for (lid, k), ctas in inst.items():
        if not all("start" in c and "end" in c for c in ctas.values()):
            continue
        d = {"id": lid, "instance": k, "kernel": names[lid], "ctas": len(ctas), "per_cta": dict(ctas)}
        for nm in _EVENTS.values():
            ts = [c[nm] for c in ctas.values() if nm in c]
            if ts:
                d[nm + "_min"] = min(ts)
                d[nm + "_max"] = max(ts)
        out.append(d)
    out.sort(key=lambda d: d["start_min"])
    return out


def chain_rows(launches: list[dict]) -> list[dict]:
    """Per launch, in microseconds: its span (first CTA start to last CTA end), the spread of
    CTA starts, how long after the previous launch's last CTA ended its consumers got past the
    dependency wait, the prologue (last wait -> last prologue end), the consumers' spread of
    ends, and, for the CTA that ended last (the one the next launch waits for), how long after
    its prologue its last weights landed and how long it computed after that."""
    rows = []
    prev = None
    for d in launches:
        us = lambda a, b: (d[a] - d[b]) / 1e3  # noqa: E731
        row = {
            "kernel": d["kernel"], "id": d["id"], "ctas": d["ctas"],
            "span": us("end_max", "start_min"),
            "start_spread": us("start_max", "start_min"),
            "prologue": us("prologue_max", "waited_max") if "prologue_max" in d else None,
            # inside the prologue: activation arrival after the wait, and the RMSNorm reduction
            "x_latency": us("xloaded_max", "waited_max") if "xloaded_max" in d else None,
            "reduce": us("reduced_max", "xall_max") if "reduced_max" in d and "xall_max" in d else None,
            "end_spread": us("end_max", "end_min"),
            "produced_before_end": us("end_max", "produced_max") if "produced_max" in d else None,
        }
        ctas = d.get("per_cta", {})
        if ctas:
            xs = [(c["xall"] - c["waited"]) / 1e3 for c in ctas.values() if "xall" in c and "waited" in c]
            if xs:
                row["mean_x_all_warps"] = float(np.mean(xs))
                row["max_x_all_warps"] = float(np.max(xs))
            qs = [(c["prologue"] - c.get("reduced", c["xall"])) / 1e3 for c in ctas.values()
                  if "xall" in c and "prologue" in c]
            if qs:
                row["mean_quantize"] = float(np.mean(qs))
            last = max(ctas.values(), key=lambda c: c["end"])
            if "prologue" in last and "last_full" in last:
                row["crit_data_after_prologue"] = (last["last_full"] - last["prologue"]) / 1e3
                row["crit_compute_after_data"] = (last["end"] - max(last["last_full"], last["prologue"])) / 1e3
                row["crit_start_to_end"] = (last["end"] - last["start"]) / 1e3
            lat = [(c["last_full"] - c["prologue"]) / 1e3 for c in ctas.values() if "last_full" in c and "prologue" in c]
            if lat:
                row["mean_data_after_prologue"] = float(np.mean(lat))
            prod = [(c["produced"] - c["start"]) / 1e3 for c in ctas.values() if "produced" in c]
            if prod:
                row["mean_producer_issue"] = float(np.mean(prod))
        if d["kernel"] == "k_attention_exact" and ctas:
            # mean duration of each phase over the heads' CTAs
            for a, b in zip(ATTN_PHASES, ATTN_PHASES[1:]):
                v = [(c[b] - c[a]) / 1e3 for c in ctas.values() if a in c and b in c]
                if v:
                    row["phase_" + b] = float(np.mean(v))
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
            "x_latency", "reduce", "start_spread", "end_spread", "produced_before_end", "crit_data_after_prologue",
            "crit_compute_after_data", "crit_start_to_end", "mean_data_after_prologue", "mean_producer_issue",
            "mean_x_all_warps", "max_x_all_warps", "mean_quantize"]
    short = ["launches", "span", "end_after_prev", "start_after_prev", "waited_after_prev", "prologue", "x_latency",
             "reduce", "start_spread", "end_spread", "produced<end", "crit_data", "crit_compute", "crit_span",
             "mean_data", "prod_issue", "x_all_mean", "x_all_max", "quantize"]
    lines = ["kernel                              " + " ".join(f"{c:>12}" for c in short)]
    for kern, f in summ.items():
        lines.append(f"{kern:36}" + " ".join(f"{f.get(c, float('nan')):12.3f}" for c in cols))
    attn = {k: f for k, f in summ.items() if k.startswith("k_attention_exact")}
    if attn:
        ph = ["phase_" + p for p in ATTN_PHASES[1:]]
        lines.append("attention phases (mean over heads, us): " + " ".join(f"{p[6:]:>9}" for p in ph))
        for kern, f in attn.items():
            lines.append(f"{kern:40}" + " ".join(f"{f.get(p, float('nan')):9.3f}" for p in ph))
    return "\n".join(lines)
