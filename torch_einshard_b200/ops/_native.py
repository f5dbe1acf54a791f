"""Loader for the in-tree sm_100a extension ``torch_einshard_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).  On a machine with a CUDA device, a missing or
broken extension is an error as soon as a native op is requested (set
``EINSHARD_ALLOW_TORCH_FALLBACK=1`` to run the torch reference path instead);
on CPU-only machines the torch path is used silently.

``EINSHARD_WAIT_TIMEOUT_US`` (default 4 s) bounds every device-side wait on a
peer rank (flag spins of the fused and collective kernels); a wait that runs
out records its code in the error word and the kernel returns.
"""

import os

import torch

__all__ = ["module", "available", "require", "error_word", "check_errors", "reset_errors", "EinshardCommTimeout",
           "set_wait_timeout_us", "wait_timeout_us"]

_state = {"loaded": False, "module": None, "error": None}
_ERROR_WORDS = {}


def module():
    if not _state["loaded"]:
        _state["loaded"] = True
        try:
            from .. import _C  # noqa: F401
            _state["module"] = _C
            env = os.environ.get("EINSHARD_WAIT_TIMEOUT_US")
            if env:
                _C.set_wait_timeout_ns(int(float(env) * 1000))
        except Exception as error:  # noqa: BLE001 - reported through require()
            _state["error"] = error
    return _state["module"]


def allow_fallback() -> bool:
    return os.environ.get("EINSHARD_ALLOW_TORCH_FALLBACK", "0") not in ("", "0")


def available() -> bool:
    return module() is not None


def require():
    mod = module()
    if mod is None:
        raise RuntimeError(
            "torch_einshard_b200 native extension is not built or failed to load "
            f"({_state['error']!r}); run `python setup.py build_ext --inplace`"
        )
    return mod


def set_wait_timeout_us(us):
    """Bound (microseconds) of device-side waits on peer ranks for kernels
    launched from now on."""
    require().set_wait_timeout_ns(max(1, int(us * 1000)))


def wait_timeout_us():
    return require().get_wait_timeout_ns() / 1000.0


def error_word(device) -> torch.Tensor:
    """Per-device int32 word that kernels set when a bounded wait gives up."""
    index = torch.device(device).index
    if index is None:
        index = torch.cuda.current_device()
    word = _ERROR_WORDS.get(index)
    if word is None:
        word = torch.zeros(4, dtype=torch.int32, device=f"cuda:{index}")
        _ERROR_WORDS[index] = word
    return word


_CODES = {
    1: "TMA stage never filled", 2: "shared-memory stage never released",
    3: "accumulator never completed", 4: "accumulator never released",
    5: "peer flag never set (a peer rank did not arrive)", 6: "drain timed out", 7: "bad arguments",
}


class EinshardCommTimeout(RuntimeError):
    """A native kernel gave up a bounded wait (a peer never arrived, a pipeline
    stage never completed).  The kernel returned cleanly; the CUDA context is
    still usable, but the op's output is invalid."""


def check_errors(device=None):
    """Raise :class:`EinshardCommTimeout` if any native kernel on ``device``
    reported a timeout (synchronises)."""
    if device is None:
        devices = list(_ERROR_WORDS)
    else:
        index = torch.device(device).index if not isinstance(device, int) else device
        devices = [torch.cuda.current_device() if index is None else index]
    for index in devices:
        word = _ERROR_WORDS.get(index)
        if word is None:
            continue
        code = int(word[0].item())
        if code:
            raise EinshardCommTimeout(f"einshard native kernel on cuda:{index} aborted: {_CODES.get(code, code)}")


def reset_errors():
    for word in _ERROR_WORDS.values():
        word.zero_()
