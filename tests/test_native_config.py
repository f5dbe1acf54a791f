"""Runtime settings of the native extension that need no GPU."""

import os
import subprocess
import sys

import pytest

from torch_einshard_b200.ops import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
needs_ext = pytest.mark.skipif(_native.module() is None, reason="native extension not built")


@needs_ext
def test_wait_timeout_setting_round_trips():
    previous = _native.wait_timeout_us()
    try:
        _native.set_wait_timeout_us(1234.5)
        assert _native.wait_timeout_us() == pytest.approx(1234.5)
        _native.set_wait_timeout_us(0)  # clamped to the smallest bound, never "wait forever"
        assert _native.wait_timeout_us() > 0
    finally:
        _native.set_wait_timeout_us(previous)


@needs_ext
def test_wait_timeout_env_is_read_at_load():
    env = dict(os.environ, EINSHARD_WAIT_TIMEOUT_US="250000", PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-c", "from torch_einshard_b200.ops import _native; "
                          "_native.module(); print(_native.wait_timeout_us())"],
                         env=env, capture_output=True, text=True, timeout=300, check=True)
    assert float(out.stdout.strip().splitlines()[-1]) == 250000.0
