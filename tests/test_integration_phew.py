"""The binding into an unchanged phew (CPU only; skipped when the phew
reference is not importable).  Runs the reference's tracer, passes and
MLXCodegen with ``phew_b200.integration.install()`` and checks the emitted
source targets this backend."""

from __future__ import annotations

import sys

import pytest

from conftest import REFERENCE, reference_importable

pytestmark = pytest.mark.skipif(not reference_importable(), reason="phew reference not importable")


@pytest.fixture(scope="module")
def phew_mod():
    sys.path.insert(0, str(REFERENCE))
    sys.path.insert(0, str(REFERENCE.parent))
    from tests.golden import make_golden  # noqa: F401  (registers the oracle as mlx.core)

    core = make_golden.fake_mlx()
    from phew_b200 import integration

    integration.install(mx_module=False)
    import phew

    return phew, core, make_golden


def test_fusion_pass_uses_cuda_emitter(phew_mod):
    phew, core, mg = phew_mod
    from phew.rules import run_all_passes

    g = mg.graphs(core)["gelu_chain"]()
    g, applied = run_all_passes(g, enable_tensorops=False, enable_fusion=True)
    assert "elementwise_fusion" in applied
    kernels = [n for n in g.nodes() if type(n).__name__ == "MetalKernel"]
    assert len(kernels) == 1
    assert "phew_h2_mul" in kernels[0].source and "phew-io:" in kernels[0].source


def test_codegen_targets_backend(phew_mod):
    phew, core, mg = phew_mod
    from phew.rules import run_all_passes

    g, _ = run_all_passes(mg.graphs(core)["rms_norm"](), enable_tensorops=False, enable_fusion=True)
    src = phew.emit.MLXCodegen().emit(g, fn_name="opt")
    assert src.startswith("import phew_b200.mx as mx\n")
    assert "mx.fast.cuda_kernel(" in src and "metal_kernel" not in src
    assert "grid=(mx.elementwise_threads(" in src
    compile(src, "<opt>", "exec")


def test_checker_and_bench_are_rebound(phew_mod):
    phew, _, _ = phew_mod
    import phew.bench
    import phew.verify

    from phew_b200 import bench, verify

    assert phew.verify.EquivalenceChecker is verify.EquivalenceChecker
    assert phew.bench.benchmark is bench.benchmark


def test_golden_sources_are_current(phew_mod):
    """The committed decoder candidates equal what the reference's passes
    emit now (regenerate with tests/golden/make_golden.py if this fails)."""
    from pathlib import Path

    phew, core, mg = phew_mod
    g, _ = mg.apply_candidate(mg.graphs(core)["decoder_tiny"](), True, False, False, True)
    src = phew.emit.MLXCodegen().emit(g, fn_name="optimized")
    ref = (Path(mg.HERE) / "sources" / "decoder_tiny__rms1_sdpa0_nmm0_fus1.py").read_text()
    strip = [ln for ln in src.splitlines() if "_kernel_" not in ln and "kernel" not in ln]
    strip_ref = [ln for ln in ref.splitlines() if "_kernel_" not in ln and "kernel" not in ln]
    assert strip == strip_ref
