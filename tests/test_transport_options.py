"""Transport options on the host, without a GPU: the step sweep's configuration
strings, the world-size defaults, and the process-wide switches that
``bench.py`` applies and reports (the library's setters only store a value,
so they run on a machine without a device)."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_stepsweep_config_strings():
    from tempname_dcu_b200.ops.stepsweep import parse_config
    assert parse_config("ag=3,epi=off,wg=40") == dict(ag=3, epi=False, wg=40)
    assert parse_config(" embx=on , rs=4 ") == dict(embx=True, rs=4)
    assert parse_config("") == {}
    with pytest.raises(ValueError, match="unknown key"):
        parse_config("tile=128")
    with pytest.raises(ValueError, match="on\\|off"):
        parse_config("epi=yes")


def test_overlap_default_follows_world_size():
    from tempname_dcu_b200.models.gpt import default_wgrad_sms
    assert default_wgrad_sms(1) == 0 and default_wgrad_sms(2) == 0
    assert default_wgrad_sms(4) == default_wgrad_sms(8) == 40


def test_bench_applies_and_reports_transport(monkeypatch):
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.remove(str(ROOT))
    from tempname_dcu_b200 import runtime
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.parallel import allgather, embedding_exchange
    before = (allgather.ag_variant(), int(native.lib().tdb_rs_set_variant(-1)), runtime.epilogue_reduction_default(),
              embedding_exchange.enabled())
    assert before == (-1, 0, False, True)  # the defaults measured fastest on 8 GPUs
    monkeypatch.setattr(sys, "argv", ["bench.py", "--ag-variant", "3", "--rs-variant", "4",
                                      "--epilogue-reduction", "on", "--embedding-exchange", "off"])
    try:
        got = bench.apply_transport(bench.parse())
        assert got == dict(ag_variant=3, rs_variant=4, epilogue_reduction=True, embedding_exchange=False)
    finally:
        allgather.set_ag_variant(before[0])
        runtime.set_rs_variant(before[1])
        runtime.set_epilogue_reduction(before[2])
        embedding_exchange.set_embedding_exchange(before[3])
    assert (allgather.ag_variant(), runtime.epilogue_reduction_default()) == (-1, False)


def test_grid_limit_is_scoped():
    from tempname_dcu_b200.ops import native
    lib = native.lib()
    assert lib.tdb_set_grid_limit(-1) == 0  # a negative value only reads
    with native.grid_limit(100):
        assert lib.tdb_set_grid_limit(-1) == 100
        with native.grid_limit(40):
            assert lib.tdb_set_grid_limit(-1) == 40
        assert lib.tdb_set_grid_limit(-1) == 100
    assert lib.tdb_set_grid_limit(-1) == 0


def test_exposed_communication_estimate_from_opbench_rows():
    from tempname_dcu_b200.models.config import BENCH_CONFIG
    from tempname_dcu_b200.ops.roofline import exposed_from_opbench
    rows = [dict(role="attn", arm="flux", world=8, fused_us=66.5, gemm_only_us=24.1),
            dict(role="attn", arm="flux_taco", world=8, fused_us=10.0, gemm_only_us=24.1),  # not a BF16 row
            dict(role="mlp", arm="flux", world=8, fused_us=80.3, gemm_only_us=31.4),
            dict(role="ag_qkv", world=8, fused_us=94.8, gemm_only_us=30.8),
            dict(role="ag_qkv", world=8, fused_us=84.8, gemm_only_us=30.8),  # the fastest form counts
            dict(role="ag_fc1", world=8, fused_us=96.7, gemm_only_us=33.2),
            dict(role="ag_fc1", world=4, fused_us=1.0, gemm_only_us=0.0)]   # another world size
    per_path, total = exposed_from_opbench(rows, BENCH_CONFIG, 8)
    per_layer = (84.8 - 30.8) * 2 + (96.7 - 33.2) * 2 + (66.5 - 24.1) + (80.3 - 31.4) * 3
    assert len(per_path) == 8
    assert abs(total - 32 * 8 * per_layer) < 1e-6
    with pytest.raises(ValueError, match="missing"):
        exposed_from_opbench(rows[:2], BENCH_CONFIG, 8)
