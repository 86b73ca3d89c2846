"""Per-step attention metadata for the mixers, engine-free.

Under vLLM the mixers read `get_forward_context().attn_metadata[prefix]`
(mixers.py:852-856); outside an engine (tests, benchmarks, the full-model
harness) the same object is installed here with `set_forward_metadata`.  The
metadata is duck-typed: any object with vLLM's Mamba2 metadata field names works.
"""

from __future__ import annotations

import contextlib
import sys
import threading

_state = threading.local()


def get_forward_metadata():
    return getattr(_state, "meta", None)


@contextlib.contextmanager
def set_forward_metadata(meta):
    prev = getattr(_state, "meta", None)
    _state.meta = meta
    try:
        yield
    finally:
        _state.meta = prev


def _vllm_metadata():
    if "vllm.forward_context" not in sys.modules:  # never import vLLM just to look
        return None
    try:
        from vllm.forward_context import get_forward_context, is_forward_context_available
    except Exception:  # vLLM absent or a different version: engine-free use only
        return None
    try:
        if not is_forward_context_available():
            return None
        return get_forward_context().attn_metadata
    except Exception:
        return None


def lookup(prefix):
    """The metadata of layer `prefix` for the current step, or None (profile run)."""
    raw = get_forward_metadata()
    if raw is None:
        raw = _vllm_metadata()
    if raw is None:
        return None
    return raw[prefix] if isinstance(raw, dict) else raw
