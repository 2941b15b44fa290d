"""Range attribution of a torch.profiler Chrome trace: for every atlas.* range, its span (wall time of
the range on the device timeline), busy time (sum of the GPU kernels that ran inside it) and its top
kernels. The same report as the reference's atlas/proftrace.py:32-81, computed from the trace's
"gpu_user_annotation" ranges (the device-side projection of record_function ranges) and its
"kernel" events; a kernel belongs to the innermost range that contains its start."""
from __future__ import annotations

import json
from collections import defaultdict
from pathlib import Path


def _events(trace) -> list:
    if isinstance(trace, (str, Path)):
        trace = json.loads(Path(trace).read_text())
    return trace.get("traceEvents", trace) if isinstance(trace, dict) else trace


def attribute(trace, prefix: str = "atlas.") -> dict:
    """{range name: {"count", "span_us", "busy_us", "idle_us", "kernels": {kernel: us}}} plus a
    "_total" entry for all kernels of the trace."""
    ev = _events(trace)
    ranges = [e for e in ev if e.get("ph") == "X" and e.get("cat") == "gpu_user_annotation"
              and str(e.get("name", "")).startswith(prefix)]
    kernels = [e for e in ev if e.get("ph") == "X" and e.get("cat") == "kernel"]
    ranges.sort(key=lambda e: (e["ts"], -e.get("dur", 0)))
    out = defaultdict(lambda: {"count": 0, "span_us": 0.0, "busy_us": 0.0, "kernels": defaultdict(float)})
    for r in ranges:
        o = out[r["name"]]
        o["count"] += 1
        o["span_us"] += float(r.get("dur", 0))
    total = {"count": len(kernels), "span_us": 0.0, "busy_us": 0.0, "kernels": defaultdict(float)}
    for k in kernels:
        t0, d = float(k["ts"]), float(k.get("dur", 0))
        total["busy_us"] += d
        total["kernels"][k["name"]] += d
        inner = None
        for r in ranges:  # innermost = the latest-starting range that still contains the kernel start
            if r["ts"] <= t0 < r["ts"] + r.get("dur", 0):
                if inner is None or r["ts"] >= inner["ts"]:
                    inner = r
            elif r["ts"] > t0:
                break
        if inner is not None:
            o = out[inner["name"]]
            o["busy_us"] += d
            o["kernels"][k["name"]] += d
    if kernels:
        total["span_us"] = max(float(k["ts"]) + float(k.get("dur", 0)) for k in kernels) - min(float(k["ts"]) for k in kernels)
    res = {}
    for name, o in list(out.items()) + [("_total", total)]:
        res[name] = {"count": o["count"], "span_us": o["span_us"], "busy_us": o["busy_us"],
                     "idle_us": max(0.0, o["span_us"] - o["busy_us"]),
                     "kernels": dict(sorted(o["kernels"].items(), key=lambda kv: -kv[1]))}
    return res


def table(res: dict, top: int = 10) -> str:
    """Plain-text report of `attribute`: one block per range, largest busy time first."""
    lines = []
    for name, o in sorted(res.items(), key=lambda kv: -kv[1]["busy_us"]):
        lines.append(f"{name:28s} n={o['count']:5d}  span {o['span_us'] / 1e3:9.3f} ms  busy {o['busy_us'] / 1e3:9.3f} ms"
                     f"  idle {o['idle_us'] / 1e3:9.3f} ms")
        for k, us in list(o["kernels"].items())[:top]:
            lines.append(f"    {us / 1e3:9.3f} ms  {k[:100]}")
    return "\n".join(lines) + "\n"
