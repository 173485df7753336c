"""Failure detection on one B200, with the failure made on the host: no GPU fault, trap or hang.

The reference reports its failures as exceptions (ValueError "KV cache full",
src/forward.nim:290-291; GQA shape, :247-248).  This path adds the failures of a split-KV group:

* a peer whose values never arrive.  TL_DIST_FAULT_SILENT_PEER=1 at tl_dist_init makes a
  one-rank group exchange as rank 0 of two, with a second rank that never posts (a message the
  test drops).  The decode kernel's wait for it is bounded (TL_DIST_WAIT_MS, here 200 ms);
  then the kernel sets the timeout bit of the device error word and returns, the call reports
  TL_ERR_DEVICE "wait-timeout", and the handle and the GPU context stay usable;
* a rank that never joins tl_dist_init.  The set-up is non-blocking and gives up after
  TL_DIST_INIT_TIMEOUT_MS with TL_ERR_NCCL.  It runs in a child process, so that a failure of
  this test cannot leave anything behind in the test process."""
import ctypes as C
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from tests.helpers import randn

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def ptr(t):
    return C.c_void_p(t.data_ptr())


class Env:
    """Set environment variables for the scope (the library reads them at tl_dist_init and,
    for TL_DECODE_CLUSTER, on every call), then put the old values back."""

    def __init__(self, **kw):
        self.kw = kw
        self.old = {}

    def __enter__(self):
        for k, v in self.kw.items():
            self.old[k] = os.environ.get(k)
            os.environ[k] = v

    def __exit__(self, *exc):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.mark.parametrize("cluster", ["1", "0"])
def test_split_kv_peer_that_never_posts_times_out(cuda_lib, cluster):
    import torch
    _lib = cuda_lib
    B, Hq, Hkv, D, L = 2, 32, 8, 128, 3000
    rng = np.random.default_rng(5)
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, 500000.0, L, B, 1, 0))
    try:
        for b in range(B):
            kk = torch.from_numpy(randn(rng, L, Hkv * D)).cuda()
            vv = torch.from_numpy(randn(rng, L, Hkv * D)).cuda()
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, ptr(kk), ptr(vv), L, None))
        q = torch.from_numpy(randn(rng, B, Hq * D)).cuda()
        pos = np.array([L - 1, L // 3], np.int32)
        dpos = torch.from_numpy(pos).cuda()
        f = pos.ctypes.data_as(C.c_void_p)
        before = torch.empty(B, Hq * D, device="cuda")
        with Env(TL_DECODE_CLUSTER=cluster):
            _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(before), None))
            _lib.check(_lib.lib.tl_check_device(h, None))
            uid = C.create_string_buffer(128)
            _lib.check(_lib.lib.tl_dist_unique_id(uid))
            with Env(TL_DIST_FAULT_SILENT_PEER="1", TL_DIST_WAIT_MS="200"):
                _lib.check(_lib.lib.tl_dist_init(h, uid, 1, 0))
            out = torch.zeros(B, Hq * D, device="cuda")
            t0 = time.perf_counter()
            rc = _lib.lib.tl_decode_attention_dist(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(out), None)
            assert rc == _lib.TL_OK, _lib.lib.tl_last_error()
            rc = _lib.lib.tl_check_device(h, None)
            waited = time.perf_counter() - t0
            assert rc == _lib.TL_ERR_DEVICE, rc
            assert b"wait-timeout" in _lib.lib.tl_last_error()
            assert 0.15 <= waited < 10.0, waited
            # the error word was read and cleared, the context is intact: the handle works on
            after = torch.empty(B, Hq * D, device="cuda")
            _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(after), None))
            _lib.check(_lib.lib.tl_check_device(h, None))
            assert torch.equal(before, after)
            # and so does the injected group: every call keeps timing out the same way
            rc = _lib.lib.tl_decode_attention_dist(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(out), None)
            assert rc == _lib.TL_OK and _lib.lib.tl_check_device(h, None) == _lib.TL_ERR_DEVICE
            _lib.check(_lib.lib.tl_dist_resync(h))
    finally:
        _lib.lib.tl_attn_destroy(h)


_NEVER_JOINS = r"""
import ctypes as C, sys, time
sys.path.insert(0, {root!r})
import torch
torch.cuda.set_device(0)
from tinylama_b200 import _lib
h = C.c_void_p()
_lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, 32, 8, 128, 128, 500000.0, 64, 1, 1, 0))
uid = C.create_string_buffer(128)
_lib.check(_lib.lib.tl_dist_unique_id(uid))
t0 = time.perf_counter()
rc = _lib.lib.tl_dist_init(h, uid, 2, 0)   # rank 1 of 2 never joins
dt = time.perf_counter() - t0
msg = _lib.lib.tl_last_error().decode()
# the handle is still usable on its own
h2 = C.c_void_p()
rc2 = _lib.lib.tl_attn_create(C.byref(h2), 1, 32, 8, 128, 128, 500000.0, 64, 1, 1, 0)
_lib.lib.tl_attn_destroy(h2)
_lib.lib.tl_attn_destroy(h)
print(f"RESULT rc={{rc}} rc2={{rc2}} dt={{dt:.2f}} msg={{msg}}", flush=True)
"""


def test_dist_init_gives_up_when_a_rank_never_joins(cuda_lib):
    env = dict(os.environ, TL_DIST_INIT_TIMEOUT_MS="3000", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS.format(root=ROOT)], env=env, capture_output=True,
                       text=True, timeout=240)
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
    assert r.returncode == 0 and line, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    fields = dict(kv.split("=", 1) for kv in line[0][len("RESULT "):].split(" ", 3))
    assert int(fields["rc"]) == cuda_lib.TL_ERR_NCCL, line[0]
    assert "did not form" in fields["msg"], line[0]
    assert 2.5 <= float(fields["dt"]) < 60.0, line[0]
    assert int(fields["rc2"]) == cuda_lib.TL_OK, line[0]
