"""Loader for the in-tree CUDA extension ``elasticmegatron_b200._C``.

CUDA tensors are only ever processed by the hand-written sm_100a kernels of this extension.  If the
extension is missing on a machine with a GPU, :func:`ext` raises instead of silently falling back to
PyTorch; CPU tensors use ``ops/reference.py``.
"""
from __future__ import annotations

import os
import threading

import torch

_EXT = None
_ERR = None
_LOCK = threading.Lock()
# Host-side count of kernel launches issued through this package (used by the benchmark's
# ``gpu_launches`` figure).  The extension increments its own counter; see :func:`launch_count`.


def ext():
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    with _LOCK:
        if _EXT is None:
            try:
                from elasticmegatron_b200 import _C  # type: ignore

                _EXT = _C
            except Exception as e:  # pragma: no cover - exercised on GPU boxes without a build
                _ERR = e
                raise RuntimeError(
                    "elasticmegatron_b200._C is not built; run `python setup.py build_ext --inplace` "
                    f"(import error: {e!r})") from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def use_native(t: torch.Tensor) -> bool:
    """True for CUDA tensors (and then the extension must exist)."""
    if t.is_cuda:
        ext()
        return True
    return False


def launch_count() -> int:
    if _EXT is None:
        return 0
    return int(_EXT.launch_count())


def reset_launch_count() -> None:
    if _EXT is not None:
        _EXT.reset_launch_count()


def so_path() -> str:
    e = ext()
    return os.path.abspath(e.__file__)


def check_device_errors() -> None:
    """Raise if a bounded device-side wait of this package's kernels gave up (GEMM pipeline barriers, attention
    pipelines, symmetric-memory barriers).  Each read is a 4-byte device->host copy, so call it where the host
    already synchronises (after reading the loss)."""
    if _EXT is None or not torch.cuda.is_available():
        return
    flags = {"gemm": _EXT.gemm_error_flag(), "comm": _EXT.comm_error_flag(),
             "attn_fwd": _EXT.attn_error_flag(), "attn_bwd": _EXT.attn_bwd_error_flag()}
    bad = {k: hex(v) for k, v in flags.items() if v}
    if bad:
        raise RuntimeError(f"device-side wait timed out (kernel error flags {bad}); results of this step are invalid")
