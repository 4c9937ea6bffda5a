"""The C-ABI library: it loads, exports every function include/tsrc.h declares, and its host-side
logic (refusal reasons, argument errors, no-device handling) works without a GPU."""
import ctypes as ct

import pytest

import tsrc


def test_exports_every_declared_symbol():
    L = tsrc.lib()
    declared = tsrc.declared_symbols()
    assert len(declared) >= 10
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    # the binding covers the whole header, and nothing more
    assert sorted(declared) == sorted(tsrc._SIGS)


def test_version():
    assert tsrc.lib().tsrc_version().decode().startswith("tsrc ")


@pytest.mark.parametrize("fmt,N,K,ok", [(0, 4864, 896, True), (1, 14336, 4096, True), (1, 10, 4000, False),
                                        (0, 10, 33, False), (2, 10, 32, False), (0, 0, 32, False),
                                        (0, 10, 65536 + 32, False), (1, 1, 65536, True)])
def test_mul_mat_refusals(fmt, N, K, ok):
    why = tsrc.mul_mat_unsupported(fmt, N, K, 1)
    assert (why is None) == ok, why
    if not ok:
        assert why.startswith("MUL_MAT")


def test_null_arguments_are_errors_not_crashes():
    L = tsrc.lib()
    assert L.tsrc_close(None) == tsrc.E_ARG
    assert b"NULL" in L.tsrc_last_error()
    assert L.tsrc_weight_free(None) == tsrc.E_ARG
    assert L.tsrc_mul_mat(None, None, None, 1, 0, None, 0, None, 0, 0, 1.0, 1.0, None) == tsrc.E_ARG
    assert L.tsrc_open(0, None) == tsrc.E_ARG
    assert L.tsrc_kv_create(None, 1, 64, 16, None) == tsrc.E_ARG
    assert L.tsrc_kv_free(None) == tsrc.E_ARG
    assert L.tsrc_kv_set_rows(None, None, 0, None, 1, 0, None, 0, None) == tsrc.E_ARG
    assert L.tsrc_kv_set_bytes(None, 0, None, 0, 1) == tsrc.E_ARG
    assert L.tsrc_kv_get_bytes(None, 0, None, 0, 1) == tsrc.E_ARG
    assert L.tsrc_flash_attn(None, None, None, 1, 4, 1, None, 0, 0.125, 0, 0, None, None, None) == tsrc.E_ARG


def test_open_without_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ct.c_void_p()
    rc = tsrc.lib().tsrc_open(0, ct.byref(h))
    assert rc == tsrc.E_NODEV and not h.value
    with pytest.raises(tsrc.TsrcError):
        tsrc.Device(0)
