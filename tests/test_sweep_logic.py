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



def test_groups_are_largest_size_first():
    g = sweep.make_groups(SEEDS[:2], SIZES, VARIANTS)
    assert len(g) == 2 * len(SIZES) * len(VARIANTS)
    assert [x.size for x in g[:8]] == ["large"] * 8
    assert g[0] == sweep.Group(0, "large", VARIANTS[0]) and g[-1].size == "small"


def test_lone_rank_runs_every_group_and_merge_folds_them(tmp_path):
    """A rank whose peers never start takes every group from the shared
    counter; the merge folds the group records into shard verdicts."""
    from torch.distributed import HashStore

    cands = CANDS[:5]
    groups = sweep.make_groups(SEEDS[:3], SIZES, VARIANTS)
    ev = fake_eval({("c1", "pm1e4")})
    recs = sweep.run_groups(groups, cands, ev, HashStore(), rank=1, journal=tmp_path / "journal.rank1.jsonl")
    assert [(r.seed, r.size, r.variant) for r in recs] == [(g.seed, g.size, g.variant) for g in groups]
    assert len(ev.calls) == len(groups) * len(cands)  # one evaluation per unit
    shards = sweep.make_shards(cands, SEEDS[:3])
    verdicts, missing = sweep.merge(tmp_path, shards, SIZES, VARIANTS)
    assert not missing
    assert {c for c, v in verdicts.items() if not v["passed"]} == {"c1"}
    assert verdicts["c1"]["shards"] == 3 and len(verdicts["c1"]["failures"]) == 3 * len(SIZES)
    assert verdicts["c1"]["failures"][0].startswith("size=small seed=0 variant=pm1e4")


def test_group_resume_and_missing_groups(tmp_path):
    from torch.distributed import HashStore

    cands = CANDS[:4]
    groups = sweep.make_groups(SEEDS[:2], SIZES, VARIANTS)
    shards = sweep.make_shards(cands, SEEDS[:2])
    # a previous run finished the first 5 groups (all large, seed 0 and one of seed 1)
    store = HashStore()
    store.add("x/next", 0)
    part = sweep.run_groups(groups[:5], cands, fake_eval(set()), store, rank=1,
                            journal=tmp_path / "journal.rank1.jsonl", run_id="x")
    assert len(part) == 5
    verdicts, missing = sweep.merge(tmp_path, shards, SIZES, VARIANTS)
    assert set(missing) == set(shards)  # no seed has all its groups yet
    assert not any(v["passed"] for v in verdicts.values())
    ev = fake_eval(set())
    recs = sweep.run_groups(groups, cands, ev, HashStore(), rank=0, journal=tmp_path / "journal.rank0.jsonl")
    assert len(recs) == len(groups)
    assert len(ev.calls) == (len(groups) - 5) * len(cands)
    verdicts, missing = sweep.merge(tmp_path, shards, SIZES, VARIANTS)
    assert not missing and all(v["passed"] for v in verdicts.values())


def _group_worker(rank, world, port, jdir, crash_rank):
    import datetime
    import time

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from torch.distributed import distributed_c10d

    store = distributed_c10d._get_default_store()
    groups = sweep.make_groups(SEEDS[:2], SIZES, VARIANTS)
    shards = sweep.make_shards(CANDS, SEEDS[:2])
    base = fake_eval({("c3", "subnormal")})

    def evaluate(cand, seed, size, variant):
        if rank == 1:  # a slower rank: the other one takes more groups
            time.sleep(0.002)
        return base(cand, seed, size, variant)

    jpath = Path(jdir) / f"journal.rank{rank}.jsonl"
    lost = None
    if rank == crash_rank:
        # take the first group, then fail before journalling it (a host-side
        # failure between steps); the others start once it holds the group
        lost = store.add("t/next", 1) - 1
        dist.barrier()
    else:
        if crash_rank is not None:
            dist.barrier()
        sweep.run_groups(groups, CANDS, evaluate, store, rank, journal=jpath, run_id="t")
    dist.barrier()
    if rank == 0:
        verdicts, missing = sweep.merge(Path(jdir), shards, SIZES, VARIANTS)
        n_missing = len(missing)
        if missing:  # the lost group's seed is open for every candidate: reassign
            sweep.run_shards(missing, evaluate, SIZES, VARIANTS, journal=jpath, rank=0)
            verdicts, missing = sweep.merge(Path(jdir), shards, SIZES, VARIANTS)
        (Path(jdir) / "result.json").write_text(json.dumps(
            {"reassigned": n_missing, "missing": len(missing),
             "passed": sorted(c for c, v in verdicts.items() if v["passed"])}))
    _ = lost
    dist.destroy_process_group()


@pytest.mark.parametrize("crash_rank", [None, 1])
def test_two_rank_gloo_group_sweep(tmp_path, crash_rank):
    port = _free_port()
    mp.spawn(_group_worker, args=(2, port, str(tmp_path), crash_rank), nprocs=2, join=True)
    res = json.loads((tmp_path / "result.json").read_text())
    assert res["missing"] == 0
    assert res["passed"] == sorted(c for c in CANDS if c != "c3")
    done = []
    for p in sorted(tmp_path.glob("journal.rank*.jsonl")):
        done += [(tuple(d["group"]), d["rank"]) for d in map(json.loads, p.read_text().splitlines())
                 if "group" in d]
    keys = [g for g, _ in done]
    assert len(keys) == len(set(keys))  # no group ran twice
    n_groups = 2 * len(SIZES) * len(VARIANTS)
    if crash_rank is None:
        assert len(keys) == n_groups and res["reassigned"] == 0
    else:
        # the held group (largest size, seed 0) never ran; its seed's shards were reassigned
        assert len(keys) == n_groups - 1 and (0, "large", VARIANTS[0]) not in keys
        assert res["reassigned"] == len(CANDS)


@pytest.mark.parametrize("depth", [1, 2])
def test_prefetch_claims_groups_ahead(depth):
    """With a prefetch hook a rank keeps `depth` groups claimed beyond the
    one it evaluates and hands each to the hook as it claims it; every
    group still runs exactly once, in list order."""
    from torch.distributed import HashStore

    cands = CANDS[:3]
    groups = sweep.make_groups(SEEDS[:2], SIZES, VARIANTS)
    events = []
    base = fake_eval(set())

    def evaluate(cand, seed, size, variant):
        events.append(("eval", (seed, size, variant)))
        return base(cand, seed, size, variant)

    def prefetch(g):
        events.append(("prefetch", (g.seed, g.size, g.variant)))

    recs = sweep.run_groups(groups, cands, evaluate, HashStore(), prefetch=prefetch,
                            prefetch_depth=depth)
    keys = [(g.seed, g.size, g.variant) for g in groups]
    assert [(r.seed, r.size, r.variant) for r in recs] == keys
    assert [k for e, k in events if e == "prefetch"] == keys
    # when group n is first evaluated, groups up to n + depth were prefetched
    for n, k in enumerate(keys):
        first_eval = events.index(("eval", k))
        seen = {kk for e, kk in events[:first_eval] if e == "prefetch"}
        assert set(keys[:min(len(keys), n + depth + 1)]) <= seen


def _prefetch_worker(rank, world, port, jdir):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from torch.distributed import distributed_c10d

    store = distributed_c10d._get_default_store()
    groups = sweep.make_groups(SEEDS[:2], SIZES, VARIANTS)
    prefetched, evaluated = [], []
    base = fake_eval(set())

    def evaluate(cand, seed, size, variant):
        if cand == CANDS[0]:
            evaluated.append([seed, size, variant])
        return base(cand, seed, size, variant)

    sweep.run_groups(groups, CANDS[:2], evaluate, store, rank,
                     journal=Path(jdir) / f"journal.rank{rank}.jsonl", run_id="p",
                     prefetch=lambda g: prefetched.append([g.seed, g.size, g.variant]))
    (Path(jdir) / f"rank{rank}.json").write_text(json.dumps({"pre": prefetched, "ev": evaluated}))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_prefetch_sweep(tmp_path):
    port = _free_port()
    mp.spawn(_prefetch_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    runs = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(2)]
    all_ev = [tuple(k) for r in runs for k in r["ev"]]
    assert len(all_ev) == len(set(all_ev)) == 2 * len(SIZES) * len(VARIANTS)
    for r in runs:
        # a rank prefetches only groups it then evaluates itself
        assert all(k in r["ev"] for k in r["pre"])
