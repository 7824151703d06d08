"""Verification sweep: phew's equivalence protocol over many candidates,
sharded across GPUs.

The reference verifies one candidate at a time in one process
(``verify/checker.py:77-218``, called from ``optimizer.py:319-322``): for
each size, seed and edge variant it evaluates baseline and candidate and
applies the allclose rule.  Here a sweep verifies a set of candidates
against one baseline:

* unit   = (candidate, seed, size, variant): one baseline/candidate pair
           compared on the device (``phew_compare``);
* group  = (seed, size, variant): every candidate's unit of it, sharing
           one baseline evaluation (the unit of scheduling, ``run_groups``);
* shard  = (candidate, seed): every size and variant of one seed (the unit
           of verdicts and of reassignment, ``run_shards``);
* verdict per candidate = all of its shards passed (one failing unit fails
  the candidate, as in the reference).

Processes (one per GPU) take groups, largest size first, from one counter
in a host-side key-value store, so the baseline of each group runs once in
the whole job and ranks finish within about one group of each other.  Each
process draws a group's inputs on its own device.  There is no data-path
collective: processes append records to per-rank journals, and the merge
folds them back into per-candidate verdicts (a rerun skips groups already
journalled, and the shards that a dead rank's missing groups leave open are
returned for reassignment).

Two variant sets:
* ``reference``: random / zeros / x1e-6 / x1e6, drawn on the host with
  ``np.random.default_rng(seed + 1000)`` exactly as the reference does
  (``verify/checker.py:235-263``); for sizes where host draws are cheap;
* ``edge``: zeros / N(0,1)*1e4 / N(0,1)*1e-39 (bf16 subnormals) / one-hot
  rows, drawn on the device by ``phew_fill`` from (seed, variant, argument).
  Like the reference's variants they replace every array argument.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Callable, Sequence

import numpy as np

VARIANT_SETS = {
    "reference": ("random", "zeros", "small_scale", "large_scale"),
    "edge": ("zeros", "pm1e4", "subnormal", "one_hot_rows"),
}
FILL_NORMAL, FILL_UNIFORM, FILL_ONE_HOT, FILL_CONSTANT = 0, 1, 2, 3


@dataclass(frozen=True)
class Shard:
    candidate: str
    seed: int


@dataclass
class ShardVerdict:
    candidate: str
    seed: int
    passed: bool
    failures: list = field(default_factory=list)
    units: int = 0
    seconds: float = 0.0
    rank: int = 0

    def to_json(self) -> str:
        return json.dumps(asdict(self))


def make_shards(candidates: Sequence[str], seeds: Sequence[int]) -> list[Shard]:
    """Seed-major order: consecutive shards share a seed (and its inputs)."""
    return [Shard(c, s) for s in seeds for c in candidates]


def partition(shards: Sequence[Shard], world: int, rank: int) -> list[Shard]:
    """Contiguous block `rank` of `world` (sizes differ by at most one)."""
    n = len(shards)
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return list(shards[lo:hi])


def _stream_id(*parts) -> int:
    h = hashlib.sha1("/".join(str(p) for p in parts).encode()).digest()
    return int.from_bytes(h[:8], "little")


# ---------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------


@dataclass
class ArgSpec:
    """One argument of the baseline: shape, dtype name and how to draw it
    ("normal" with std 1/sqrt(fan_in), "ones", "causal_mask")."""

    shape: tuple
    dtype: str
    kind: str = "normal"
    fan_in: int = 1


class DeviceInputs:
    """Seeded device arrays for the baseline's arguments and their variants."""

    def __init__(self, arg_specs: Callable[[str], list[ArgSpec]]) -> None:
        self.arg_specs = arg_specs

    def _fill(self, shape, dtype, kind, seed, stream, scale):
        from . import _native
        from .mx.core import _stream, empty

        out = empty(shape, dtype)
        cols = shape[-1] if len(shape) else 1
        _native.call("phew_fill", ctypes.c_void_p(out._t.data_ptr()), out.size, max(cols, 1),
                     out.dtype.code, kind, ctypes.c_uint64(seed & (2**64 - 1)),
                     ctypes.c_uint64(stream), ctypes.c_float(scale), _stream())
        return out

    def base(self, size: str, seed: int) -> list:
        from .mx.core import array
        from .ops import causal_mask

        from . import dtypes as dt

        args = []
        for i, spec in enumerate(self.arg_specs(size)):
            if spec.kind == "ones":
                args.append(self._fill(spec.shape, spec.dtype, FILL_CONSTANT, 0, 0, 1.0))
            elif spec.kind == "causal_mask":
                L, S = spec.shape[-2], spec.shape[-1]
                args.append(causal_mask(L, S, dt.from_any(spec.dtype)))
            else:
                scale = 1.0 / float(np.sqrt(spec.fan_in))
                args.append(self._fill(spec.shape, spec.dtype, FILL_NORMAL, seed,
                                       _stream_id("base", size, i), scale))
        _ = array
        return args

    def variant(self, name: str, base_args: list, size: str, seed: int) -> list:
        from .mx.core import array, zeros_like

        if name == "random":
            return base_args
        if name == "zeros":
            return [zeros_like(a) for a in base_args]
        if name in ("small_scale", "large_scale"):
            # reference draws (host): verify/checker.py:246-263
            rng = np.random.default_rng(seed + 1000)
            small = [array(rng.standard_normal(a.shape).astype(np.float32) * 1e-6).astype(a.dtype)
                     for a in base_args]
            if name == "small_scale":
                return small
            return [array(rng.standard_normal(a.shape).astype(np.float32) * 1e6).astype(a.dtype)
                    for a in base_args]
        kinds = {"pm1e4": (FILL_NORMAL, 1e4), "subnormal": (FILL_NORMAL, 1e-39),
                 "one_hot_rows": (FILL_ONE_HOT, 1.0)}
        if name not in kinds:
            raise ValueError(f"unknown variant {name!r}")
        kind, scale = kinds[name]
        return [self._fill(a.shape, a.dtype, kind, seed, _stream_id(name, size, i), scale)
                for i, a in enumerate(base_args)]


class HostInputs:
    """The inputs of `DeviceInputs`, drawn on the HOST and copied in.

    The reference's input factories and edge variants draw on the host
    (``examples/rms_norm.py:27-31``, ``verify/checker.py:235-263``) and
    hand the arrays to the device.  This provider does the same at sweep
    scale: ``phew_fill_host`` runs the counter-based generator of
    ``phew_fill`` on host threads into pinned buffers, and every group's
    arguments are copied host -> device before the group is evaluated.
    With ``prefetch(group)`` upcoming groups are drawn on a background
    thread, in order, while the device evaluates earlier ones (`slots`
    pinned buffers used round robin: a prefetch depth of d needs d + 1; a
    slot is redrawn only after the copies out of it have finished).  The
    thread that draws a group also issues its host -> device copies, on a
    stream of their own, so they overlap the compute of the groups before
    it; the compute stream waits for a group's copies only when it reaches
    that group.

    Variants: the edge set (zeros, pm1e4, subnormal, one_hot_rows) and the
    base draw ("random"), with the arguments `DeviceInputs` gives them.
    ``h2d_bytes`` counts the bytes copied in."""

    def __init__(self, arg_specs: Callable[[str], list[ArgSpec]], sizes: Sequence[str],
                 threads: int = 0, slots: int = 2) -> None:
        import threading

        import torch

        self.arg_specs = arg_specs
        self.threads = threads
        self.h2d_bytes = 0
        self._lock = threading.Lock()
        self._pending: dict[tuple, Any] = {}
        self._slot = 0
        self._device = torch.cuda.current_device()
        # one pinned buffer per argument and slot, sized for the largest size
        cap = [0] * len(arg_specs(sizes[0]))
        for z in sizes:
            for j, a in enumerate(arg_specs(z)):
                cap[j] = max(cap[j], int(np.prod(a.shape)) * _itemsize(a.dtype))
        self._slots = max(2, int(slots))
        self._pinned = [[torch.empty(c, dtype=torch.uint8).pin_memory() for c in cap]
                        for _ in range(self._slots)]
        self._copied = [None] * self._slots  # event: copies out of the slot have finished
        self._copy_stream = torch.cuda.Stream(device=self._device)
        self._pool = None

    # -- host side ---------------------------------------------------------
    def _draw(self, slot: int, seed: int, size: str, variant: str) -> tuple:
        """Draw one group's arguments into pinned slot `slot` and copy them
        to the device on the copy stream.  Returns (device tensors, the
        event that marks the copies done, bytes copied)."""
        import torch

        from . import _native
        from . import dtypes as dt

        ev = self._copied[slot]
        if ev is not None:
            ev.synchronize()
        out = []
        for i, spec in enumerate(self.arg_specs(size)):
            n = int(np.prod(spec.shape))
            d = dt.from_any(spec.dtype)
            buf = self._pinned[slot][i][: n * _itemsize(spec.dtype)]
            ptr = ctypes.c_void_p(buf.data_ptr())
            cols = max(spec.shape[-1] if len(spec.shape) else 1, 1)

            def fill(kind, stream, scale):
                _native.call("phew_fill_host", ptr, ctypes.c_int64(n), ctypes.c_int64(cols),
                             d.code, kind, ctypes.c_uint64(seed & (2**64 - 1)),
                             ctypes.c_uint64(stream), ctypes.c_float(scale), self.threads)

            if variant == "zeros":
                buf.zero_()
            elif variant == "random":
                if spec.kind == "ones":
                    fill(FILL_CONSTANT, 0, 1.0)
                elif spec.kind == "causal_mask":
                    L, S = spec.shape[-2], spec.shape[-1]
                    m = np.zeros((L, S), np.float32)
                    m[np.triu_indices(L, S - L + 1, S)] = -np.inf
                    buf.numpy()[:] = np.frombuffer(m.astype(d.np).tobytes(), np.uint8)
                else:
                    fill(FILL_NORMAL, _stream_id("base", size, i), 1.0 / float(np.sqrt(spec.fan_in)))
            else:
                kinds = {"pm1e4": (FILL_NORMAL, 1e4), "subnormal": (FILL_NORMAL, 1e-39),
                         "one_hot_rows": (FILL_ONE_HOT, 1.0)}
                if variant not in kinds:
                    raise ValueError(f"HostInputs: variant {variant!r} is not drawn on the host")
                kind, scale = kinds[variant]
                fill(kind, _stream_id(variant, size, i), scale)
            out.append((buf, spec))
        tensors, nbytes = [], 0
        with torch.cuda.device(self._device), torch.cuda.stream(self._copy_stream):
            for buf, spec in out:
                t = torch.empty(spec.shape, dtype=dt.from_any(spec.dtype).torch, device=self._device)
                t.view(torch.uint8).view(-1).copy_(buf, non_blocking=True)
                tensors.append(t)
                nbytes += buf.numel()
            done = torch.cuda.Event()
            done.record(self._copy_stream)
        self._copied[slot] = done  # only this slot's next draw (same thread or caller) reads it
        return tensors, done, nbytes

    def prefetch(self, group: Group) -> None:
        """Start drawing `group`'s arguments on a background thread."""
        import concurrent.futures as cf

        if self._pool is None:
            self._pool = cf.ThreadPoolExecutor(max_workers=1)
        with self._lock:
            key = (group.seed, group.size, group.variant)
            if key in self._pending:
                return
            slot = self._slot
            self._slot = (self._slot + 1) % self._slots
            self._pending[key] = (slot, self._pool.submit(self._draw, slot, *key))

    # -- the DeviceInputs interface ----------------------------------------
    def base(self, size: str, seed: int) -> list:
        return list(self.arg_specs(size))

    def variant(self, name: str, base_args: list, size: str, seed: int) -> list:
        import torch

        from .mx.core import array

        key = (seed, size, name)
        with self._lock:
            hit = self._pending.pop(key, None)
            if hit is None:
                slot = self._slot
                self._slot = (self._slot + 1) % self._slots
        if hit is not None:
            slot, fut = hit
            tensors, done, nbytes = fut.result()
        else:
            tensors, done, nbytes = self._draw(slot, seed, size, name)
        cur = torch.cuda.current_stream(self._device)
        cur.wait_event(done)
        for t in tensors:
            t.record_stream(cur)  # allocated on the copy stream, used on this one
        self.h2d_bytes += nbytes
        return [array(t) for t in tensors]

    def close(self) -> None:
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None


def _itemsize(dtype_name: str) -> int:
    return {"float32": 4, "float16": 2, "bfloat16": 2}[dtype_name]


# ---------------------------------------------------------------------------
# running shards
# ---------------------------------------------------------------------------


def load_journal(path: Path) -> dict[tuple, ShardVerdict]:
    done = {}
    if path.exists():
        for line in path.read_text().splitlines():
            if line.strip():
                d = json.loads(line)
                if "group" not in d:
                    done[(d["candidate"], d["seed"])] = ShardVerdict(**d)
    return done


def run_shards(
    shards: Sequence[Shard],
    evaluate: Callable[[str, int, str, str], tuple[bool, str | None]],
    sizes: Sequence[str],
    variants: Sequence[str],
    journal: Path | None = None,
    rank: int = 0,
    on_group: Callable[[int, str], None] | None = None,
) -> list[ShardVerdict]:
    """Run `shards` in order.  `evaluate(candidate, seed, size, variant)`
    returns (ok, failure string or None) for one unit.  Shards already in
    `journal` are skipped (resume); each finished shard is appended to it."""
    done = load_journal(journal) if journal else {}
    out = []
    by_seed: dict[int, list[Shard]] = {}
    for s in shards:
        by_seed.setdefault(s.seed, []).append(s)
    for seed, group in by_seed.items():
        todo = [s for s in group if (s.candidate, s.seed) not in done]
        out += [done[(s.candidate, s.seed)] for s in group if (s.candidate, s.seed) in done]
        if not todo:
            continue
        verdicts = {s.candidate: ShardVerdict(s.candidate, seed, True, rank=rank) for s in todo}
        t0 = time.perf_counter()
        for size in sizes:
            if on_group:
                on_group(seed, size)
            for variant in variants:
                for s in todo:
                    ok, failure = evaluate(s.candidate, seed, size, variant)
                    v = verdicts[s.candidate]
                    v.units += 1
                    if not ok:
                        v.passed = False
                        v.failures.append(failure)
        dt = time.perf_counter() - t0
        for s in todo:
            v = verdicts[s.candidate]
            v.seconds = dt / len(todo)
            out.append(v)
            if journal:
                with open(journal, "a") as f:
                    f.write(v.to_json() + "\n")
    return out


@dataclass(frozen=True)
class Group:
    """Every candidate's unit of one (seed, size, variant): the baseline runs
    once for the whole group."""

    seed: int
    size: str
    variant: str


@dataclass
class GroupRecord:
    seed: int
    size: str
    variant: str
    results: dict = field(default_factory=dict)  # candidate -> failure string, or None if it passed
    seconds: float = 0.0
    rank: int = 0

    def to_json(self) -> str:
        return json.dumps({"group": [self.seed, self.size, self.variant], "results": self.results,
                           "seconds": self.seconds, "rank": self.rank})


def make_groups(seeds: Sequence[int], sizes: Sequence[str], variants: Sequence[str]) -> list[Group]:
    """Largest size first (`sizes` runs smallest to largest; cost grows with
    it), then seed, then variant: taken in this order from one shared queue
    the groups form a longest-processing-time-first list schedule."""
    return [Group(seed, size, v) for size in reversed(sizes) for seed in seeds for v in variants]


def load_groups(path: Path) -> dict[tuple, GroupRecord]:
    done = {}
    if path.exists():
        for line in path.read_text().splitlines():
            if line.strip():
                d = json.loads(line)
                if "group" in d:
                    seed, size, variant = d["group"]
                    done[(seed, size, variant)] = GroupRecord(seed, size, variant, d["results"],
                                                              d["seconds"], d["rank"])
    return done


def run_groups(
    groups: Sequence[Group],
    candidates: Sequence[str],
    evaluate: Callable[[str, int, str, str], tuple[bool, str | None]],
    store: Any,
    rank: int = 0,
    journal: Path | None = None,
    run_id: str = "sweep",
    prefetch: Callable[[Group], None] | None = None,
    prefetch_depth: int = 1,
) -> list[GroupRecord]:
    """Evaluate groups taken from one shared counter, in list order, until
    the list is exhausted.

    The next group is ``store.add(f"{run_id}/next", 1) - 1``; `store` is any
    key-value store with an atomic ``add`` (torch.distributed's TCP / file /
    hash store): host control only, no device data moves between ranks.  A
    group costs one baseline plus every candidate, and a rank that is free
    takes the next one, so ranks finish within about one group of each other
    and no baseline is computed twice.  Groups already journalled (by any
    rank: every ``*.jsonl`` beside `journal` is read) are not re-evaluated;
    each finished group is appended to `journal`.

    With `prefetch`, a rank keeps `prefetch_depth` groups claimed beyond the
    one it is evaluating and calls ``prefetch(group)`` as it claims each, so
    that preparing their inputs (a host-side draw) overlaps the device work
    of the groups before them."""
    from collections import deque

    done: dict[tuple, GroupRecord] = {}
    if journal:
        for p in sorted(Path(journal).parent.glob("*.jsonl")):
            done.update(load_groups(p))
    out: list[GroupRecord] = []
    key = f"{run_id}/next"
    ahead = max(1, int(prefetch_depth)) if prefetch is not None else 0

    def claim() -> int:
        i = store.add(key, 1) - 1
        if prefetch is not None and i < len(groups):
            g = groups[i]
            if (g.seed, g.size, g.variant) not in done:
                prefetch(g)
        return i

    queue = deque([claim()])
    while queue and queue[0] < len(groups):
        while len(queue) < 1 + ahead and queue[-1] < len(groups):
            queue.append(claim())
        i = queue.popleft()
        g = groups[i]
        k = (g.seed, g.size, g.variant)
        if k in done:
            out.append(done[k])
        else:
            t0 = time.perf_counter()
            rec = GroupRecord(g.seed, g.size, g.variant, rank=rank)
            for c in candidates:
                ok, failure = evaluate(c, g.seed, g.size, g.variant)
                rec.results[c] = None if ok else failure
            rec.seconds = time.perf_counter() - t0
            out.append(rec)
            if journal:
                with open(journal, "a") as f:
                    f.write(rec.to_json() + "\n")
        if not queue:
            queue.append(claim())
    return out


def merge(journal_dir: Path, shards: Sequence[Shard], sizes: Sequence[str] = (),
          variants: Sequence[str] = ()) -> tuple[dict[str, dict], list[Shard]]:
    """Per-candidate verdicts from every rank's journal, plus the shards no
    journal holds (to be reassigned).  Group records count towards a shard
    (candidate, seed) once the groups of all `sizes` x `variants` of its seed
    are journalled."""
    recs: dict[tuple, ShardVerdict] = {}
    groups: dict[tuple, GroupRecord] = {}
    for p in sorted(Path(journal_dir).glob("journal.rank*.jsonl")):
        recs.update(load_journal(p))
        groups.update(load_groups(p))
    if groups:
        for sh in shards:
            if (sh.candidate, sh.seed) in recs:
                continue
            found = [groups.get((sh.seed, z, v)) for z in sizes for v in variants]
            if not found or any(g is None or sh.candidate not in g.results for g in found):
                continue
            fails = [g.results[sh.candidate] for g in found if g.results[sh.candidate] is not None]
            recs[(sh.candidate, sh.seed)] = ShardVerdict(
                sh.candidate, sh.seed, not fails, fails, len(found),
                sum(g.seconds for g in found) / max(len(g.results) for g in found), found[0].rank)
    missing = [s for s in shards if (s.candidate, s.seed) not in recs]
    cands: dict[str, dict] = {}
    for s in shards:
        c = cands.setdefault(s.candidate, {"passed": True, "failures": [], "shards": 0})
        r = recs.get((s.candidate, s.seed))
        if r is None:
            c["passed"] = False
            continue
        c["shards"] += 1
        c["passed"] = c["passed"] and r.passed
        c["failures"] += r.failures
    return cands, missing


# ---------------------------------------------------------------------------
# device evaluation of one unit
# ---------------------------------------------------------------------------


class DeviceEvaluator:
    """Evaluates units on the current GPU, caching the baseline output and
    the inputs of the current (seed, size, variant)."""

    def __init__(self, baseline: Callable, candidates: dict[str, Callable], inputs: DeviceInputs,
                 checker=None) -> None:
        from .verify import EquivalenceChecker

        self.baseline = baseline
        self.candidates = candidates
        self.inputs = inputs
        self.checker = checker or EquivalenceChecker()
        self._key = None
        self._base_args = None
        self._args = None
        self._base_out = None
        self._base_exc = None

    def _prepare(self, seed: int, size: str, variant: str) -> None:
        key = (seed, size, variant)
        if key == self._key:
            return
        self._args = self._base_out = self._base_exc = None
        if self._key is None or self._key[:2] != (seed, size):
            self._base_args = None
            self._base_args = self.inputs.base(size, seed)
        self._args = self.inputs.variant(variant, self._base_args, size, seed)
        try:
            self._base_out = self.baseline(*self._args)
        except Exception as exc:  # noqa: BLE001
            self._base_exc = exc
        self._key = key

    def __call__(self, candidate: str, seed: int, size: str, variant: str):
        self._prepare(seed, size, variant)
        tag = f"size={size} seed={seed} variant={variant}"
        try:
            if self._base_exc is not None:
                raise self._base_exc
            out = self.candidates[candidate](*self._args)
            ok, max_diff = self.checker.check_unit(self._base_out, out)
            if ok:
                return True, None
            return False, f"{tag} max_diff={max_diff:.3e}"
        except Exception as exc:  # noqa: BLE001  (the reference records any failure)
            return False, f"{tag} exception={exc}"

    def release(self) -> None:
        self._key = self._base_args = self._args = self._base_out = None


def load_candidates(sources: dict[str, str]) -> dict[str, Callable]:
    """exec() each emitted ``output_source`` (as ``optimizer.py:365-369``
    does) and return its ``optimized`` function."""
    out = {}
    for name, src in sources.items():
        ns: dict[str, Any] = {}
        exec(compile(src, f"<{name}>", "exec"), ns)
        out[name] = ns["optimized"]
    return out


def env_rank() -> tuple[int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
