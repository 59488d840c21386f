"""Exposed-communication accounting of a profiled step (synthetic timelines)."""

from nanospec_b200.utils.trace import kernel_events, overlap_summary


def _ev(cat, name, ts, dur, stream):
    return {"cat": cat, "name": name, "ts": ts, "dur": dur, "args": {"stream": stream}}


def test_copy_engine_transfers_count_as_communication():
    events = [
        # compute stream 7: three kernels with a gap [30, 40)
        _ev("kernel", "gemm_bf16_kernel", 0, 10, 7), _ev("kernel", "attn_fwd_kernel", 10, 20, 7),
        _ev("kernel", "adamw_kernel", 40, 20, 7),
        # a local copy on the compute stream is compute, not communication
        _ev("gpu_memcpy", "Memcpy DtoD (Device -> Device)", 30, 2, 7),
        # communication stream 21: a peer copy half hidden, a reduce kernel fully exposed
        _ev("gpu_memcpy", "Memcpy PtoP (Device -> Device)", 20, 20, 21),
        _ev("kernel", "ns::local_reduce_avg_kernel", 60, 5, 21),
        _ev("kernel", "ns::peer_wait_kernel", 65, 1, 21),
    ]
    s = overlap_summary(kernel_events(events))
    # comm union: [20, 40) + [60, 66) = 26 us; hidden: [20, 30) under attention and
    # [30, 32) under the compute-stream copy = 12 us
    assert s["comm_us"] == 26
    assert s["hidden_us"] == 12
    assert s["exposed_comm_us"] == 14
    assert {r["kernel"] for r in s["kernels"]} == {"memcpy:Memcpy PtoP (Device -> Device)",
                                                   "ns::local_reduce_avg_kernel", "ns::peer_wait_kernel"}
