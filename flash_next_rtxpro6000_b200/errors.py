"""Device-side error reporting.

Every wait inside the kernels is bounded: a wait that runs out of time records an error
code in its workspace's ``error_flag`` (the first code of a call wins), the kernel leaves
its loop and the launch completes, so the CUDA context stays usable, but that call's
outputs are wrong.  The launch itself reports success; the flag is how the host learns
of it.  Nothing on the device clears a flag.

``check_device_errors`` reads every flag this process has created (the dense GEMV
scratch slots, every MoE workspace from ``make_workspace``) in one device-to-host copy,
clears the ones that are set and raises ``DeviceWaitError`` naming them.  It
synchronises the current stream, so call it outside CUDA graph capture, after the work
whose results you are about to trust (for example once per decode step, or in tests).
"""

from __future__ import annotations

import threading
import weakref
from typing import List, Optional, Tuple

import torch

from ._lib import DEVICE_ERRORS


class DeviceWaitError(RuntimeError):
    """A kernel's bounded wait ran out of time; ``codes`` lists (source, code) pairs."""

    def __init__(self, codes: List[Tuple[str, int]]):
        self.codes = codes
        msg = "; ".join(f"{src}: code {c} ({DEVICE_ERRORS.get(c, 'unknown')})" for src, c in codes)
        super().__init__("device-side wait expired, results of the affected calls are invalid: "
                         + msg)


_lock = threading.Lock()
_flags: List[Tuple["weakref.ref", str]] = []


def register(flag: torch.Tensor, source: str) -> None:
    """Track a [1] int32 device error flag (held weakly: a freed workspace drops out)."""
    with _lock:
        _flags.append((weakref.ref(flag), source))


def _live(device: Optional[torch.device]):
    out, keep = [], []
    with _lock:
        for ref, src in _flags:
            t = ref()
            if t is None:
                continue
            keep.append((ref, src))
            if device is None or t.device == device:
                out.append((t, src))
        _flags[:] = keep
    return out


def read_flags(flags, clear: bool = True) -> List[Tuple[str, int]]:
    """(source, code) of every set flag among ``flags`` [(tensor, source)], read with one
    copy per device; the set ones are cleared on the current stream when ``clear``."""
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        raise RuntimeError("device error flags cannot be read inside CUDA graph capture")
    bad = []
    by_dev = {}
    for t, src in flags:
        by_dev.setdefault(t.device, []).append((t, src))
    for dev, items in by_dev.items():
        vals = torch.cat([t.reshape(-1)[:1] for t, _ in items]).cpu().tolist()
        for (t, src), v in zip(items, vals):
            if v != 0:
                bad.append((src, int(v)))
                if clear:
                    t.zero_()
    return bad


def check_device_errors(device=None, clear: bool = True) -> None:
    """Raise DeviceWaitError if any tracked error flag (on ``device``, or on every device)
    is set; set flags are cleared first when ``clear``."""
    d = None if device is None else torch.device(device)
    if d is not None and d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    bad = read_flags(_live(d), clear=clear)
    if bad:
        raise DeviceWaitError(bad)


def check_flag(flag: torch.Tensor, source: str, clear: bool = True) -> None:
    """check_device_errors for one flag."""
    bad = read_flags([(flag, source)], clear=clear)
    if bad:
        raise DeviceWaitError(bad)
