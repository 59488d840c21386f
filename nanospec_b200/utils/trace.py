"""Device-timeline analysis: which communication time is hidden under compute.

Reference method (experiments/overlap.py:150-178): classify kernels of one
profiled step as communication or compute by name; for every communication kernel,
the union of its intersections with compute kernels on *other* streams is the
hidden part. Here the communication set also contains this project's peer kernels
(``peer_allgather``, ``peer_reduce_avg``, ``peer_wait``), and the summary adds the
*exposed* communication time: the part of the union of communication intervals not
covered by any compute kernel.
"""

from __future__ import annotations

COMM_MARKERS = ("nccl", "peer_allgather", "peer_reduce", "peer_wait", "peer_signal")


def _union(spans):
    out = []
    for lo, hi in sorted(spans):
        if out and lo <= out[-1][1]:
            out[-1][1] = max(out[-1][1], hi)
        else:
            out.append([lo, hi])
    return out


def _length(spans):
    return sum(hi - lo for lo, hi in spans)


def _intersect(a, b):
    """Length of the intersection of two unions of disjoint sorted intervals."""
    i = j = 0
    total = 0.0
    while i < len(a) and j < len(b):
        lo = max(a[i][0], b[j][0])
        hi = min(a[i][1], b[j][1])
        if hi > lo:
            total += hi - lo
        if a[i][1] < b[j][1]:
            i += 1
        else:
            j += 1
    return total


def kernel_events(trace_events):
    """(name, start_us, end_us, stream) of the GPU kernels in a Chrome trace event list."""
    out = []
    for e in trace_events:
        if e.get("cat") == "kernel" and "dur" in e:
            out.append((e.get("name", ""), float(e["ts"]), float(e["ts"]) + float(e["dur"]),
                        e.get("args", {}).get("stream")))
    return out


def is_comm(name: str) -> bool:
    low = name.lower()
    return any(m in low for m in COMM_MARKERS)


def overlap_summary(kernels):
    """Per-communication-kernel hidden time plus totals (microseconds)."""
    comm = [k for k in kernels if is_comm(k[0])]
    compute = [k for k in kernels if not is_comm(k[0])]
    rows = []
    for name, lo, hi, stream in comm:
        spans = _union([(max(lo, c[1]), min(hi, c[2])) for c in compute
                        if c[3] != stream and c[1] < hi and lo < c[2]])
        rows.append({"kernel": name, "duration_us": hi - lo, "compute_overlap_us": _length(spans)})
    comm_u = _union([(k[1], k[2]) for k in comm])
    comp_u = _union([(k[1], k[2]) for k in compute])
    comm_total = _length(comm_u)
    hidden = _intersect(comm_u, comp_u)
    span = (max(k[2] for k in kernels) - min(k[1] for k in kernels)) if kernels else 0.0
    return {
        "kernels": rows,
        "comm_us": comm_total,
        "hidden_us": hidden,
        "exposed_comm_us": comm_total - hidden,
        "compute_busy_us": _length(comp_u),
        "span_us": span,
    }
