"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, reports shapes/status strings, and builds RoPE tables that
match the restatement of src/convert.rs:161-176 bit for bit."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import qora_mixer as qm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_mixer.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|int64_t|void\*|const char\*)\s+(qm_\w+)\(", txt, re.M)))


def test_header_and_binding_list_agree():
    assert header_symbols() == sorted(qm.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = qm.lib()
    missing = [s for s in header_symbols() if not hasattr(L, s)]
    assert not missing, missing


def test_shape_matches_reference_config():
    s = qm.shape()
    # src/config.rs:56-66
    assert (s.num_qk_heads, s.num_v_heads, s.dn_head_dim, s.conv_kernel) == (16, 32, 128, 4)
    assert (s.num_attn_heads, s.num_kv_heads, s.attn_head_dim, s.rope_dim) == (16, 4, 256, 64)
    assert s.rope_theta == np.float32(1e7) and s.rms_eps == np.float32(1e-6)


def test_status_strings():
    L = qm.lib()
    assert L.qm_status_string(0) == b"ok"
    for code in range(1, 11):
        assert L.qm_status_string(code) not in (b"", b"unknown status")


def test_rope_table_bit_exact_vs_restatement(orc):
    cos, sin = qm.rope_table(1.0e7, 64, 33000)
    ocos, osin = orc.rope_table(1.0e7, 64, 33000)
    np.testing.assert_array_equal(cos, ocos)
    np.testing.assert_array_equal(sin, osin)


def test_null_arguments_are_errors_not_crashes():
    L = qm.lib()
    assert L.qm_ctx_create(0, None) == 1  # QM_E_ARG
    assert L.qm_sync(None) == 1
    assert L.qm_dn_state_destroy(None) == 1
    assert L.qm_kv_destroy(None) == 1
    assert L.qm_rope_table(C.c_float(1e7), 63, 10, None, None) == 1
    assert L.qm_dn_state_conv_pos(None) == -1
    assert L.qm_kv_seq_len(None) == -1


def test_ctx_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = qm.lib().qm_ctx_create(0, C.byref(h))
    assert rc != 0 and not h.value
