"""Meta-device construction of a strategy's training state.

The reference monkey-patches tensor factories so Megatron's ``setup_model_and_optimizer`` builds a zero-memory
model on the ``meta`` device; inter-process mode uses it to pre-plan and warm communicators before the real
state arrives (elastic_megatron/megatron_manager/meta_device_context.py:40-248).  Here the training core
already separates structure from storage, so the context only flips a flag: ``TrainingState`` objects built
inside it hold ``meta`` parameter views and no arenas, and ``rebuild()`` later gives them real memory.
"""
from __future__ import annotations

import contextlib

_META = False


@contextlib.contextmanager
def meta_device_context():
    global _META
    old = _META
    _META = True
    try:
        yield
    finally:
        _META = old


def in_meta_context() -> bool:
    return _META
