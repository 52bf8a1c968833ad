"""The harness-shaped command line over the six call sites (correctness + benchmark modes)."""
import pytest

from ggemm_asm_b200 import sites


def test_site_table_matches_the_harness_shapes():
    assert set(sites.GROUPS["all"]) == set(sites.SITES)
    assert sites.GROUPS["all_fwd"] == ["gate_up_fwd", "down_fwd", "down_dgrad", "gate_up_dgrad"]
    assert sites.GROUPS["all_wgrad"] == ["down_wgrad", "gate_up_wgrad"]
    assert sites.SITES["gate_up_dgrad"][3] == dict(K=5760, N=2880)
    assert sites.SITES["gate_up_wgrad"][3] == dict(OUT_M=2880, OUT_N=5760)


def test_unknown_site_is_an_error():
    with pytest.raises(SystemExit):
        sites.main(["--site", "nope"])


@pytest.mark.gpu
def test_all_sites_pass_the_harness_rule():
    assert sites.correctness(sites.GROUPS["all"], M=16384)


@pytest.mark.gpu
def test_benchmark_rows():
    rows = sites.benchmark(["down_fwd", "down_wgrad"], warmup=1, iters=2, M=16384)
    assert len(rows) == 2 and all(r[2] > 0 for r in rows)
