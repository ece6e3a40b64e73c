"""Host logic of the decode step's per-op accounting (SectionTimer): device
times and algorithmic bytes summed per named op, per kind, heaviest first.
CUDA events are replaced by stand-ins that report fixed elapsed times."""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "vk-shei_b200"))

from mslim_b200 import model as mdl  # noqa: E402


class _Ev:
    def __init__(self, t):
        self.t = t

    def elapsed_time(self, other):
        return other.t - self.t


def _mark(timer, kind, op, nbytes, ms, kernel=None, link="hbm"):
    sec = mdl._Section(timer, kind, op, nbytes, kernel or op, link)
    timer.marks.append((sec, _Ev(0.0), _Ev(ms)))


def test_per_op_sums_launches_time_and_bytes():
    timer = mdl.SectionTimer(torch=None)
    for _ in range(32):
        _mark(timer, "gemm", "gate|up projection", 235_012_096, 0.040, "cuBLAS GEMM")
        _mark(timer, "attention", "decode attention", 269_000_000, 0.045, "mslim_decode_split")
        _mark(timer, "collective", "NVLink reduce + residual + RMSNorm", 65_536, 0.010,
              "mslim_tp_allreduce_rmsnorm", "nvlink")
    _mark(timer, "gemm", "lm_head", 1_050_673_152, 0.160, "cuBLAS GEMM")
    ops = timer.per_op()
    # 32 x 45 us, 32 x 40 us, 32 x 10 us, 1 x 160 us
    assert [e["op"] for e in ops] == ["decode attention", "gate|up projection",
                                      "NVLink reduce + residual + RMSNorm", "lm_head"]
    by = {e["op"]: e for e in ops}
    assert by["gate|up projection"]["launches"] == 32
    assert abs(by["gate|up projection"]["ms"] - 32 * 0.040) < 1e-9
    assert by["gate|up projection"]["bytes"] == 32 * 235_012_096
    assert by["NVLink reduce + residual + RMSNorm"]["link"] == "nvlink"
    assert by["lm_head"]["kernel"] == "cuBLAS GEMM"
    kinds = timer.totals_ms()
    assert abs(kinds["gemm"] - (32 * 0.040 + 0.160)) < 1e-9
    assert abs(kinds["collective"] - 32 * 0.010) < 1e-9


def test_section_defaults_name_the_kind():
    timer = mdl.SectionTimer(torch=None)
    sec = timer("elementwise")
    assert (sec.kind, sec.op, sec.kernel, sec.nbytes, sec.link) == ("elementwise", "elementwise", "elementwise",
                                                                      0, "hbm")


def test_interleave_gate_up_layout():
    """Blocks of 64 gate rows, each followed by the up rows of the same 64
    features (the weight layout of mslim_cuda_gemv_swiglu)."""
    import pytest
    import torch
    from mslim_b200 import attention as att
    width, k = 192, 8
    gate = torch.arange(width * k, dtype=torch.int32).reshape(width, k)
    up = -gate - 1
    w = att.interleave_gate_up(gate, up)
    assert w.shape == (2 * width, k)
    for b in range(width // 64):
        assert torch.equal(w[128 * b:128 * b + 64], gate[64 * b:64 * b + 64])
        assert torch.equal(w[128 * b + 64:128 * b + 128], up[64 * b:64 * b + 64])
    with pytest.raises(att.ShapeMismatch):
        att.interleave_gate_up(gate[:100], up[:100])
