"""Installs the B200 backend into Tila's runtime (the drop-in boundary).

The reference dispatches every checked launch through two methods of
``tila.runtime._Launcher`` (runtime.py:1041-1130):

* ``_resolve_target`` imports Triton and pins the RTX 3090 target;
* ``_execute`` lowers to Triton for CUDA tensors and runs the NumPy
  interpreter for CPU arrays.

``install()`` replaces both for CUDA tensors: the target becomes a B200
``Capability`` (sm_100a, same grid/tile/dot limits, target.py:8-24) and
execution goes to :mod:`tila_b200.backend`.  CPU arrays and CPU tensors keep
the reference interpreter unchanged; every contract check, proof and race
analysis in ``_Launcher._call`` (runtime.py:726-1039) runs before either.
Triton is never imported on the B200 path.
"""

from __future__ import annotations

import os

from ._reference import tila

_target = tila.target
_runtime = tila.runtime
TilaError = tila.errors.TilaError

B200 = _target.Capability(
    name="NVIDIA B200", arch=(10, 0), triton_version="none (B200 native backend)",
    grid_limits=((1 << 31) - 1, 65535, 65535), num_warps=(4, 8),
    max_tile_elements=1 << 20, dot_inputs=("f16",), dot_outputs=("f16", "f32"),
    min_dot_k=16, fp8_storage=False, atomic_add_dtypes=("i32", "u32", "f32"),
    atomic_orders=("relaxed",), atomic_scopes=("gpu",))

_installed = None


def resolve_b200(torch, device):
    """The B200 counterpart of target.resolve_cuda (target.py:51-57)."""
    props = torch.cuda.get_device_properties(device)
    if (props.major, props.minor) != B200.arch:
        raise TilaError("TILA-TARGET-007",
                        f"unvalidated CUDA target {props.name} (sm_{props.major}{props.minor}); "
                        "the B200 backend requires sm_100")
    return _target.CUDATarget(device.index if device.index is not None else torch.cuda.current_device(),
                              str(props.uuid), torch.__version__, torch.version.cuda, B200)


def _is_cuda_launch(tensors):
    torch = _runtime.torch
    t0 = next(iter(tensors.values()), None)
    return torch is not None and isinstance(t0, torch.Tensor) and t0.is_cuda


def install():
    """Route CUDA launches of every ``@ti.jit`` kernel to the B200 backend."""
    global _installed
    if _installed is not None:
        return
    L = _runtime._Launcher
    original = (L._resolve_target, L._execute)

    def _resolve_target(self, tensors):
        if not _is_cuda_launch(tensors):
            return None
        if os.environ.get("TILA_INTERP") == "1":
            raise TilaError("TILA-TARGET-005", "CUDA tensor cannot use the forced CPU interpreter")
        return resolve_b200(_runtime.torch, next(iter(tensors.values())).device)

    def _execute(self, tensors, scalar_vals, stride_vals, consts, grid):
        if _is_cuda_launch(tensors) and os.environ.get("TILA_INTERP") != "1":
            from . import backend
            return backend.execute(self, tensors, scalar_vals, stride_vals, consts, grid)
        return original[1](self, tensors, scalar_vals, stride_vals, consts, grid)

    L._resolve_target = _resolve_target
    L._execute = _execute
    _installed = original


def uninstall():
    global _installed
    if _installed is None:
        return
    L = _runtime._Launcher
    L._resolve_target, L._execute = _installed
    _installed = None


def installed() -> bool:
    return _installed is not None
