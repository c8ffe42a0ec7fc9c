"""Step-trace breakdown: categories, per-stream busy / idle, gzip input."""
import gzip
import json

from shift_b200.analysis.step_trace import analyze, category


def test_breakdown_of_a_synthetic_two_stream_trace(tmp_path):
    ev = [
        {"ph": "X", "cat": "kernel", "name": "void sb::gemm::gemm_kernel<256>", "ts": 0, "dur": 100, "tid": 7},
        {"ph": "X", "cat": "kernel", "name": "sb::fa::fwd_kernel", "ts": 150, "dur": 50, "tid": 7},
        {"ph": "X", "cat": "kernel", "name": "sb::coll::fused_reduce_adamw_kernel<2>", "ts": 120, "dur": 200,
         "tid": 9},
        {"ph": "X", "cat": "kernel", "name": "sb::coll::flag_wait_kernel", "ts": 200, "dur": 30, "tid": 7},
        {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "ts": 0, "dur": 999, "tid": 1},
    ]
    with gzip.open(tmp_path / "trace_n2_r1.json.gz", "wt") as f:
        json.dump({"traceEvents": ev}, f)
    res = analyze(tmp_path)["rank1"]
    assert res["n_gpus"] == 2 and res["kernels"] == 4
    assert res["step_span_ms"] == 0.32
    cats = res["busy_ms_by_category"]
    assert cats["gemm"] == 0.1 and cats["attention"] == 0.05 and cats["k1_reduce_adamw"] == 0.2
    assert cats["flag_wait"] == 0.03
    s7 = res["streams"]["7"]
    assert s7["busy_ms"] == 0.18 and s7["span_ms"] == 0.23 and s7["idle_ms"] == 0.05
    assert category("ncclDevKernel_SendRecv") == "nccl"
