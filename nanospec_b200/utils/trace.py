"""Device-timeline analysis: which communication time is hidden under compute.

Reference method (experiments/overlap.py:150-178): classify kernels of one
profiled step as communication or compute by name; for every communication kernel,
the union of its intersections with compute kernels on *other* streams is the
hidden part. Here the communication set also contains this project's peer kernels
(``peer_allgather``, ``peer_reduce_avg``, ``local_reduce_avg``, ``peer_wait``) and
the copy-engine transfers of the peer schedule (memcpy activity on any stream other
than the compute stream, which is the stream with the most kernels). The summary
adds the *exposed* communication time: the part of the union of communication
intervals not covered by any compute kernel.
"""

from __future__ import annotations

COMM_MARKERS = ("nccl", "peer_allgather", "peer_reduce", "local_reduce_avg", "peer_wait", "peer_signal")
MEMCPY = "memcpy:"  # name prefix of copy-engine activity in kernel_events


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
    """(name, start_us, end_us, stream) of the GPU kernels and memcpys in a Chrome trace
    event list; memcpy names carry the ``memcpy:`` prefix."""
    out = []
    for e in trace_events:
        cat = e.get("cat")
        if cat in ("kernel", "gpu_memcpy") and "dur" in e:
            name = e.get("name", "")
            out.append(((MEMCPY + name) if cat == "gpu_memcpy" else name, float(e["ts"]),
                        float(e["ts"]) + float(e["dur"]), e.get("args", {}).get("stream")))
    return out


def is_comm(name: str) -> bool:
    low = name.lower()
    return any(m in low for m in COMM_MARKERS)


def overlap_summary(kernels):
    """Per-communication-kernel hidden time plus totals (microseconds)."""
    counts = {}
    for k in kernels:
        if not k[0].startswith(MEMCPY):
            counts[k[3]] = counts.get(k[3], 0) + 1
    main = max(counts, key=counts.get) if counts else None

    def comm_like(k):
        return is_comm(k[0]) or (k[0].startswith(MEMCPY) and k[3] != main)

    comm = [k for k in kernels if comm_like(k)]
    compute = [k for k in kernels if not comm_like(k)]
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
