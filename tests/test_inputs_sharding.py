"""CPU tests of the host logic: problem generators and expert sharding (incl. 2 gloo ranks)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ggemm_asm_b200 import inputs, sharding


def test_tiny_config_is_the_baseline_one():
    p = inputs.make_problem("tiny", seed=0)
    assert p.offs.tolist() == [0, 256, 256, 768, 1024]
    assert tuple(p.lhs.shape) == (1024, 64) and tuple(p.rhs.shape) == (1024, 128)
    assert p.lhs.dtype == torch.float8_e4m3fn and p.rhs.dtype == torch.float8_e5m2
    # amax scaling: the largest |code| hits (close to) the format maximum
    assert float(p.lhs.float().abs().max()) == 448.0
    assert float(p.rhs.float().abs().max()) == 57344.0


@pytest.mark.parametrize("name", ["gate_up", "down", "skew", "shard120b"])
def test_config_routing(name):
    cfg = inputs.CONFIGS[name]
    lens = inputs.config_lens(name, seed=0)
    assert lens.size == cfg["G"] and int(lens.sum()) == cfg["M_total"]
    assert (lens >= 0).all()
    if name == "skew":
        assert int((lens == 0).sum()) == 4
        nz = lens[lens > 0]
        assert (nz % 128 != 0).all()
        assert nz.max() > 4 * nz.mean()   # genuinely skewed
    else:
        assert (lens > 0).all()
    assert np.array_equal(lens, inputs.config_lens(name, seed=0))   # seeded


def test_per_group_scales_from_slice_amax():
    p = inputs.make_problem("skew", seed=3, G=8, M_total=2000, OUT_M=32, OUT_N=48)
    for g in range(p.G):
        lo, hi = int(p.offs[g]), int(p.offs[g + 1])
        if hi > lo:
            assert float(p.lhs[lo:hi].float().abs().max()) == 448.0
            assert float(p.rhs[lo:hi].float().abs().max()) == 57344.0
        else:
            assert float(p.lhs_scale[g]) == 1.0


def test_row_range_matches_full_problem():
    full = inputs.make_problem("tiny", seed=9, lens=[5000, 0, 12000, 3000], OUT_M=32, OUT_N=48)
    part = inputs.make_problem("tiny", seed=9, lens=[5000, 0, 12000, 3000], OUT_M=32, OUT_N=48,
                               rows=(5000, 17000))
    assert torch.equal(part.lhs.view(torch.uint8), full.lhs[5000:17000].view(torch.uint8))
    assert torch.equal(part.rhs.view(torch.uint8), full.rhs[5000:17000].view(torch.uint8))
    assert torch.equal(part.lhs_scale, full.lhs_scale)


def test_launcher_problem_matches_launcher_cpp():
    p = inputs.launcher_problem("gate_up_wgrad", G=32, M_total=131072)
    assert p.offs.tolist() == [131072 * i // 32 for i in range(33)]
    assert int(p.lhs.view(torch.uint8).unique().item()) == 0x38
    assert float(p.lhs_scale) == pytest.approx(0.1)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("name", ["gate_up", "skew", "shard120b"])
def test_partition_balanced_and_complete(name, world):
    lens = inputs.config_lens(name, seed=0)
    shards = sharding.partition(lens, world)
    assert shards[0].g_begin == 0 and shards[-1].g_end == lens.size
    for a, b in zip(shards, shards[1:]):
        assert a.g_end == b.g_begin and a.t_end == b.t_begin
    assert all(s.groups >= 1 for s in shards)
    assert sum(s.tokens for s in shards) == int(lens.sum())
    if name != "skew":
        assert sharding.imbalance(lens, shards) < 1.05 + 0.15 * (world >= 8 and lens.size <= 32)


def test_partition_more_ranks_than_groups():
    shards = sharding.partition([10, 20], 4)
    assert [s.groups for s in shards].count(0) == 2
    assert sum(s.tokens for s in shards) == 30


def test_local_offsets_rebased():
    offs = inputs.offsets_from_lens([3, 0, 5, 7])
    s = sharding.partition([3, 0, 5, 7], 2)[1]
    loc = sharding.local_offsets(offs, s)
    assert loc[0] == 0 and loc[-1] == s.tokens


def _rank_main(rank, world, port, result_q):
    """One expert-sharded rank: builds only its token slice, computes its C shard with the
    CPU oracle (stand-in for the GPU kernel on this CPU box), and gathers for validation."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        from oracle import vark_oracle as vo

        lens = [300, 0, 129, 1000, 64, 0, 511]
        full_offs = inputs.offsets_from_lens(lens)
        sh = sharding.partition(lens, world)[rank]
        part = inputs.make_problem("tiny", seed=5, lens=lens, OUT_M=16, OUT_N=32,
                                   rows=(sh.t_begin, sh.t_end))
        loc = torch.from_numpy(sharding.local_offsets(full_offs, sh))
        c = vo.wgrad_torch(part.lhs, part.rhs, part.lhs_scale, part.rhs_scale, loc)
        shapes = [None] * world
        dist.all_gather_object(shapes, (sh.g_begin, sh.g_end, c.view(torch.int16).numpy()))
        if rank == 0:
            full = inputs.make_problem("tiny", seed=5, lens=lens, OUT_M=16, OUT_N=32)
            ref = vo.wgrad_torch(full.lhs, full.rhs, full.lhs_scale, full.rhs_scale,
                                 full.group_offs).view(torch.int16).numpy()
            got = np.concatenate([s[2] for s in sorted(shapes, key=lambda s: s[0])], axis=0)
            result_q.put(bool(np.array_equal(got, ref)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    assert all(pr.exitcode == 0 for pr in procs)
    assert q.get(timeout=5) is True


def _rank_dies_main(rank, world, port, result_q):
    """Rank 1 leaves before the barrier (as a crashed rank would); rank 0 must get an error from
    the process-group timeout instead of waiting forever."""
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # no barrier, no destroy: the rank is gone
    try:
        dist.barrier()
        result_q.put("no error")
    except Exception as e:  # timeout / connection closed
        result_q.put(type(e).__name__)


def test_lost_rank_is_detected_by_the_others():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_dies_main, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=60)
    alive = [pr for pr in procs if pr.is_alive()]
    for pr in alive:
        pr.kill()
    assert not alive, "a rank hung waiting for the lost rank"
    assert q.get(timeout=5) != "no error"
