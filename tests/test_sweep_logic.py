"""Host logic of the verification sweep (CPU only): sharding, journals,
resume, merge, reassignment after a failed rank, and a 2-rank gloo run."""

from __future__ import annotations

import json
import os
import socket
from pathlib import Path

import pytest
import torch.multiprocessing as mp

from phew_b200 import sweep

CANDS = [f"c{i}" for i in range(16)]
SEEDS = list(range(5))
SIZES = ["small", "typical", "large"]
VARIANTS = sweep.VARIANT_SETS["edge"]


def fake_eval(fail_on: set):
    calls = []

    def evaluate(cand, seed, size, variant):
        calls.append((cand, seed, size, variant))
        if (cand, variant) in fail_on:
            return False, f"size={size} seed={seed} variant={variant} max_diff=1.000e+00"
        return True, None

    evaluate.calls = calls
    return evaluate


def test_shards_are_seed_major_and_partition_covers_all():
    shards = sweep.make_shards(CANDS, SEEDS)
    assert len(shards) == 80
    assert [s.seed for s in shards[:16]] == [0] * 16
    for world in (1, 2, 3, 4, 8):
        parts = [sweep.partition(shards, world, r) for r in range(world)]
        flat = [s for p in parts for s in p]
        assert flat == shards  # contiguous blocks in order
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1
        # each rank touches at most ceil(16 * 5 / world / 16) + 1 seeds
        for p in parts:
            assert len({s.seed for s in p}) <= -(-len(p) // 16) + 1


def test_run_shards_verdicts_and_unit_count(tmp_path):
    shards = sweep.make_shards(CANDS[:4], SEEDS[:2])
    ev = fake_eval({("c1", "pm1e4")})
    recs = sweep.run_shards(shards, ev, SIZES, VARIANTS, journal=tmp_path / "journal.rank0.jsonl")
    assert len(recs) == 8
    assert all(r.units == len(SIZES) * len(VARIANTS) for r in recs)
    bad = [r for r in recs if not r.passed]
    assert {(r.candidate, r.seed) for r in bad} == {("c1", 0), ("c1", 1)}
    assert bad[0].failures[0].startswith("size=small seed=0 variant=pm1e4")
    # per (seed, size, variant) the candidates run back to back (baseline reuse)
    first = ev.calls[:4]
    assert {c[1:] for c in first} == {(0, "small", "zeros")}


def test_journal_resume_skips_finished_shards(tmp_path):
    j = tmp_path / "journal.rank0.jsonl"
    shards = sweep.make_shards(CANDS[:3], SEEDS[:2])
    sweep.run_shards(shards[:3], fake_eval(set()), SIZES, VARIANTS, journal=j)
    ev = fake_eval(set())
    recs = sweep.run_shards(shards, ev, SIZES, VARIANTS, journal=j)
    assert len(recs) == 6
    assert {c[1] for c in ev.calls} == {1}  # seed 0 came from the journal
    lines = j.read_text().splitlines()
    assert len(lines) == 6 and all(json.loads(x)["passed"] for x in lines)


def test_merge_reports_missing_shards_for_reassignment(tmp_path):
    shards = sweep.make_shards(CANDS[:4], SEEDS[:2])
    sweep.run_shards(sweep.partition(shards, 2, 0), fake_eval(set()), SIZES, VARIANTS,
                     journal=tmp_path / "journal.rank0.jsonl")
    # rank 1 died before writing anything
    verdicts, missing = sweep.merge(tmp_path, shards)
    assert missing == sweep.partition(shards, 2, 1)
    assert not verdicts["c0"]["passed"]  # incomplete candidates do not pass
    # reassign the missing shards to a survivor, then everything is verified
    sweep.run_shards(missing, fake_eval(set()), SIZES, VARIANTS,
                     journal=tmp_path / "journal.rank0.jsonl")
    verdicts, missing = sweep.merge(tmp_path, shards)
    assert not missing and all(v["passed"] for v in verdicts.values())


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, jdir, crash_rank):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    shards = sweep.make_shards(CANDS, SEEDS)
    mine = sweep.partition(shards, world, rank)
    ev = fake_eval({("c3", "subnormal")})
    if rank == crash_rank:
        # fail after the first seed group: the rank reports on the host and
        # leaves between steps (no device work in flight)
        n = sum(1 for s in mine if s.seed == mine[0].seed)
        sweep.run_shards(mine[:n], ev, SIZES, VARIANTS,
                         journal=Path(jdir) / f"journal.rank{rank}.jsonl", rank=rank)
    else:
        sweep.run_shards(mine, ev, SIZES, VARIANTS,
                         journal=Path(jdir) / f"journal.rank{rank}.jsonl", rank=rank)
    dist.barrier()
    if rank == 0:
        verdicts, missing = sweep.merge(Path(jdir), shards)
        if missing:
            sweep.run_shards(missing, ev, SIZES, VARIANTS,
                             journal=Path(jdir) / "journal.rank0.jsonl", rank=0)
            verdicts, missing = sweep.merge(Path(jdir), shards)
        (Path(jdir) / "result.json").write_text(json.dumps(
            {"missing": len(missing), "passed": sorted(c for c, v in verdicts.items() if v["passed"])}))
    dist.destroy_process_group()


@pytest.mark.parametrize("crash_rank", [None, 1])
def test_two_rank_gloo_sweep(tmp_path, crash_rank):
    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path), crash_rank), nprocs=2, join=True)
    res = json.loads((tmp_path / "result.json").read_text())
    assert res["missing"] == 0
    assert res["passed"] == sorted(c for c in CANDS if c != "c3")


def _journaled(jdir: Path) -> list[tuple]:
    out = []
    for p in sorted(jdir.glob("journal.rank*.jsonl")):
        out += [(d["candidate"], d["seed"], d["rank"]) for d in map(json.loads, p.read_text().splitlines())]
    return out


def test_dynamic_lone_rank_drains_every_block(tmp_path):
    """A rank whose peers never start takes every block's shards from the
    shared counters, each exactly once."""
    from torch.distributed import HashStore

    shards = sweep.make_shards(CANDS[:5], SEEDS[:3])
    recs = sweep.run_shards_dynamic(shards, fake_eval(set()), SIZES, VARIANTS, HashStore(), rank=1,
                                    world=3, journal=tmp_path / "journal.rank1.jsonl")
    assert sorted((r.candidate, r.seed) for r in recs) == sorted((s.candidate, s.seed) for s in shards)
    # own block first, then the others
    assert [(r.candidate, r.seed) for r in recs[:5]] == [(s.candidate, s.seed) for s in sweep.partition(shards, 3, 1)]
    verdicts, missing = sweep.merge(tmp_path, shards)
    assert not missing and all(v["passed"] for v in verdicts.values())


def test_dynamic_resume_reads_every_rank_journal(tmp_path):
    from torch.distributed import HashStore

    shards = sweep.make_shards(CANDS[:4], SEEDS[:2])
    # a previous run: rank 1 finished the first three shards, then stopped
    sweep.run_shards(shards[:3], fake_eval(set()), SIZES, VARIANTS,
                     journal=tmp_path / "journal.rank1.jsonl", rank=1)
    ev = fake_eval(set())
    recs = sweep.run_shards_dynamic(shards, ev, SIZES, VARIANTS, HashStore(), rank=0, world=2,
                                    journal=tmp_path / "journal.rank0.jsonl")
    assert len(recs) == len(shards)
    assert {(c[0], c[1]) for c in ev.calls} == {(s.candidate, s.seed) for s in shards[3:]}
    assert len(_journaled(tmp_path)) == len(shards)


def _dyn_worker(rank, world, port, jdir):
    import datetime
    import time

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from torch.distributed import distributed_c10d

    store = distributed_c10d._get_default_store()
    shards = sweep.make_shards(CANDS, SEEDS[:2])
    base = fake_eval({("c3", "subnormal")})

    def evaluate(cand, seed, size, variant):
        # the second half of the shards (rank 1's block) is 20x as costly
        if seed == 1 and size == "small" and variant == VARIANTS[0]:
            time.sleep(0.04)
        return base(cand, seed, size, variant)

    sweep.run_shards_dynamic(shards, evaluate, SIZES, VARIANTS, store, rank, world,
                             journal=Path(jdir) / f"journal.rank{rank}.jsonl", run_id="t")
    dist.barrier()
    if rank == 0:
        verdicts, missing = sweep.merge(Path(jdir), shards)
        (Path(jdir) / "result.json").write_text(json.dumps(
            {"missing": len(missing), "passed": sorted(c for c, v in verdicts.items() if v["passed"])}))
    dist.destroy_process_group()


def test_two_rank_gloo_dynamic_sweep(tmp_path):
    port = _free_port()
    mp.spawn(_dyn_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    res = json.loads((tmp_path / "result.json").read_text())
    assert res["missing"] == 0
    assert res["passed"] == sorted(c for c in CANDS if c != "c3")
    done = _journaled(tmp_path)
    keys = [(c, s) for c, s, _ in done]
    assert len(keys) == len(set(keys)) == 32  # every shard exactly once
    # rank 0 finished its cheap block and took shards of rank 1's costly one
    assert any(r == 0 and s == 1 for _, s, r in done)
