"""Failure detection on the GPU without a fault.

Every device-side wait of the library is bounded (mbar_wait_bounded in
csrc/qm_ptx.cuh): when its limit passes, the waiting thread sets the error
word's timeout bit and the CTA's abort flag, the other waiters return at once,
and the kernel ends normally.  The test-only library runs that wait on a
barrier nothing arrives at, with a limit of about a millisecond, and checks
the outcome; then the GPU is used again through the product library to show
the context survived.  No trap, no fault, no hang: the wait ends by itself.
"""
import ctypes as C
import os

import pytest

import refmath
from gpu_util import dev, host, make_ctx

pytestmark = pytest.mark.gpu

LIMIT = 2_000_000  # cycles, about 1 ms


def test_bounded_wait_gives_up_and_reports():
    import qora_mixer as qm

    qm.lib()  # the self-test library links against the product library
    L = C.CDLL(os.path.join(qm.PKG_DIR, "libqora_selftest.so"))
    fn = L.qm_selftest_wait_timeout
    fn.argtypes = [C.c_longlong, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_longlong)]
    fn.restype = C.c_int
    err, n_true, longest = C.c_int(0), C.c_int(-1), C.c_longlong(0)
    rc = fn(LIMIT, C.byref(err), C.byref(n_true), C.byref(longest))
    assert rc == 0  # the kernel ended normally
    assert err.value & 1  # the timeout bit (kErrTimeout)
    assert n_true.value == 0  # no wait claimed success
    # the first waiter gave up after the limit; the abort flag released the rest
    assert LIMIT <= longest.value < 20 * LIMIT, longest.value


def test_gpu_usable_after_a_timeout():
    """After the bounded wait ran out, a DeltaNet decode through the product
    library still matches the restatement."""
    import qora_mixer as qm
    from oracle import oracle as orc
    from qora_mixer import inputs as I

    qm.lib()
    L = C.CDLL(os.path.join(qm.PKG_DIR, "libqora_selftest.so"))
    fn = L.qm_selftest_wait_timeout
    fn.argtypes = [C.c_longlong, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_longlong)]
    fn.restype = C.c_int
    err, n_true, longest = C.c_int(0), C.c_int(-1), C.c_longlong(0)
    assert fn(LIMIT, C.byref(err), C.byref(n_true), C.byref(longest)) == 0

    import torch

    ctx = make_ctx()
    try:
        c = orc.cfg_4b()
        g = I.rng(77)
        p = I.dn_layer_params(g)
        toks = I.dn_token_inputs(g, 1, 1)
        keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
        st = qm.DnState(ctx, 1)
        y = torch.empty(1, 32, 128, device="cuda")
        qm.Mixer(ctx).dn_decode(qm.dn_params(*keep), st, dev(toks["qkv"][:, 0]), dev(toks["a"][:, 0]),
                                dev(toks["b"][:, 0]), y)
        ctx.sync()  # the context's own error word is clean
        ost = orc.DnState(c)
        ref = orc.dn_decode(c, ost, toks["qkv"][0, 0], toks["a"][0, 0], toks["b"][0, 0], p["conv_w"],
                            p["a_log"], p["dt_bias"])
        assert refmath.rel_err(host(y)[0], ref) <= 1e-3
        st.close()
    finally:
        ctx.close()
