"""Small runtime helpers shared by the host wrappers: device/stream plumbing and
the optional device error word.

Device-side error reporting: every kernel can OR FI_DEVERR_* bits into a caller
int32. Reading it needs a stream synchronisation, so it is off by default; set
``FAST_INFER_B200_CHECK=1`` (or call ``set_device_checks(True)``) to have every
wrapper allocate the word, synchronise after the launch and raise on a set bit.
"""

from __future__ import annotations

import contextlib
import os

import torch

from fast_infer_b200 import _lib

_checks = os.environ.get("FAST_INFER_B200_CHECK", "0") == "1"


def set_device_checks(enabled: bool) -> None:
    global _checks
    _checks = bool(enabled)


def device_checks_enabled() -> bool:
    return _checks


def with_device(device: torch.device):
    if device.type != "cuda":
        raise ValueError("fast_infer_b200 runs on CUDA devices only")
    return torch.cuda.device(device)


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def error_word(device: torch.device):
    return torch.zeros(1, dtype=torch.int32, device=device) if _checks else None


def device_errors(word, what: str) -> None:
    if word is None:
        return
    bits = int(word.item())  # synchronises the stream
    if bits == 0:
        return
    names = []
    if bits & _lib.FI_DEVERR_TIMEOUT:
        names.append("pipeline wait timed out")
    if bits & _lib.FI_DEVERR_BAD_BLOCK:
        names.append("block_table entry outside the page pool")
    if bits & _lib.FI_DEVERR_CONTEXT_LEN:
        names.append("context length beyond max_context_len / block table")
    raise RuntimeError(f"{what}: device reported: {', '.join(names) or bits}")


@contextlib.contextmanager
def device_checks(enabled: bool = True):
    prev = _checks
    set_device_checks(enabled)
    try:
        yield
    finally:
        set_device_checks(prev)
