"""The drop-in boundary: the B200 target and the execute hook."""

import numpy as np
import pytest

import tila_b200
from tila_b200 import plugin, workloads as W

ti = tila_b200.tila


def test_installed_on_import():
    assert tila_b200.installed()


def test_b200_capability_matches_the_reference_limits():
    ref = ti.target.SUPPORTED
    cap = plugin.B200
    assert cap.arch == (10, 0)
    assert cap.grid_limits == ref.grid_limits
    assert cap.max_tile_elements == ref.max_tile_elements
    assert cap.dot_inputs == ref.dot_inputs and cap.dot_outputs == ref.dot_outputs
    assert cap.min_dot_k == ref.min_dot_k


def test_cpu_arrays_still_run_on_the_interpreter():
    x = np.arange(300, dtype=np.float32)
    out = np.zeros_like(x)
    W.add_kernel[(ti.cdiv(300, 128),)](x, x, out, BLOCK=128)
    np.testing.assert_array_equal(out, x + x)


def test_uninstall_restores_the_reference_methods():
    L = ti.runtime._Launcher
    ours = (L._resolve_target, L._execute)
    tila_b200.uninstall()
    try:
        assert (L._resolve_target, L._execute) != ours
    finally:
        tila_b200.install()
    assert tila_b200.installed()


def test_non_sm100_device_is_rejected():
    class Props:
        major, minor, name, uuid = 8, 6, "NVIDIA GeForce RTX 3090", "x"

    class FakeCuda:
        @staticmethod
        def get_device_properties(device):
            return Props()

    class FakeTorch:
        cuda = FakeCuda()
        __version__ = "x"
        version = type("v", (), {"cuda": "12.8"})

    class Dev:
        index = 0
    with pytest.raises(ti.errors.TilaError) as exc:
        plugin.resolve_b200(FakeTorch, Dev())
    assert exc.value.code == "TILA-TARGET-007"


def test_resource_failures_produce_the_reference_artifact(tmp_path, monkeypatch):
    from tila_b200 import backend
    monkeypatch.setenv("TILA_BACKEND_ARTIFACTS", str(tmp_path))
    err = backend._failure(RuntimeError("threads"), "resources", "// src", {"kernel": "k"},
                           resource=("threads", 2048, 1024))
    assert err.code == "TILA-TARGET-011"
    assert err.backend_artifact and (tmp_path / err.backend_artifact).exists()


def test_build_cli_writes_cuda_tir_and_source_map(tmp_path):
    """python -m tila_b200 build: the generated CUDA, the TIR exactly as
    `tila build` writes it, a line map back to the Tila source, the cubin."""
    import json
    import semantics_support as S
    from tila_b200.__main__ import main
    from tila import cli as tila_cli
    S.binary_program(tmp_path, "f32", "+")
    src = next(tmp_path.glob("sem_bin_f32_add.py"))
    out = tmp_path / "b200"
    assert main(["build", str(src), "-o", str(out), "--cubin"]) == 0
    cu = (out / "kernel.cu").read_text()
    assert 'extern "C" __global__' in cu and "// @tila-line" in cu
    smap = json.loads((out / "kernel.map.json").read_text())
    assert smap["cuda_line_to_tila_line"] and (out / "kernel.cubin").stat().st_size > 0
    ref = tmp_path / "ref"
    assert tila_cli.main(["build", str(src), "-o", str(ref)]) == 0
    assert (out / "kernel.tir.txt").read_text() == (ref / "kernel.tir.txt").read_text()


def test_build_cli_emits_the_launch_time_tensor_core_plan(tmp_path):
    """The build-time facts (contiguous, 16-byte aligned rows) give the
    reference matmul example the TMA ring and tcgen05 MMAs a launch gets."""
    from tila_b200._reference import reference_tree
    from tila_b200.__main__ import main
    src = reference_tree() / "examples" / "matmul.py"
    assert main(["build", str(src), "-o", str(tmp_path), "--const", "BM=128", "--const", "BN=128",
                 "--const", "BK=64"]) == 0
    cu = (tmp_path / "matmul_kernel.cu").read_text()
    assert "tila::tma_load_2d(" in cu and "tila::mma_f16_ss(" in cu


@pytest.mark.parametrize("example,consts", [
    ("add_kernel.py", ["BLOCK=1024"]),
    ("softmax.py", ["BN=1024"]),
    ("matmul.py", ["BM=128", "BN=128", "BK=64"]),
    ("fused_attention.py", ["CAUSAL=0", "BM=128", "BN=128", "BD=128"]),
    ("fused_attention.py", ["CAUSAL=1", "BM=128", "BN=128", "BD=128"]),
    ("self_attention.py", ["BM=128", "BN=128", "BD=64"]),
])
def test_every_reference_example_builds_to_an_sm100a_cubin(tmp_path, example, consts):
    """Each Tila kernel the reference ships in examples/ (the benchmarked
    configurations) generates CUDA that NVRTC compiles for sm_100a, with no
    GPU present: a code-generation regression fails here before any launch."""
    from tila_b200._reference import reference_tree
    from tila_b200.__main__ import main
    src = reference_tree() / "examples" / example
    args = ["build", str(src), "-o", str(tmp_path), "--cubin"]
    for c in consts:
        args += ["--const", c]
    assert main(args) == 0
    cubins = list(tmp_path.glob("*.cubin"))
    assert cubins and all(c.stat().st_size > 0 for c in cubins)


def test_repeated_signature_key_follows_every_tila_switch(monkeypatch):
    """The repeated-signature path keys on every TILA_* variable (TILA_SAFETY,
    TILA_RACE_MAX_PAIRS and TILA_PROOF_* included): flipping one makes the
    next launch run the full checks."""
    monkeypatch.setenv("TILA_SAFETY", "strict")
    before = plugin._tila_env()
    monkeypatch.setenv("TILA_SAFETY", "warn")
    assert plugin._tila_env() != before
    for name in ("TILA_RACE_MAX_PAIRS", "TILA_PROOF_TIMEOUT_MS"):
        key = plugin._tila_env()
        monkeypatch.setenv(name, "7")
        assert plugin._tila_env() != key


def test_replaced_statement_invalidates_the_repeated_signature_path():
    from dataclasses import replace
    jf = ti.jit(W.add_kernel.fn)
    stmts = tuple(plugin._statements(jf.tk.body, []))
    assert plugin._same_tir(jf.tk, jf.tk, stmts)
    store = jf.tk.body[-1]
    jf.tk.body[-1] = replace(store)
    assert not plugin._same_tir(jf.tk, jf.tk, stmts)
