"""The C ABI library loads and exports every entry point include/w4b200.h declares;
host-side validation rejects bad arguments before touching a GPU."""
import ctypes
import re

import pytest

from roofline_decoding_b200 import _lib


def declared_functions():
    text = _lib.HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w4_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for must in ("w4_pack", "w4_dequant", "w4_gemv", "w4_gemv_ex", "w4_gemv_default_config",
                 "w4_init", "w4_version", "w4_status_string", "w4_last_error",
                 "w4_device_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in w4b200.h but not exported"
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version_and_status_strings():
    lib = _lib.load()
    text = _lib.HEADER_PATH.read_text()
    version = int(re.search(r"#define W4B200_VERSION (\d+)", text).group(1))
    assert lib.w4_version() == version
    assert lib.w4_status_string(0) == b"W4_OK"
    assert lib.w4_status_string(1) == b"W4_ERR_INVALID_ARG"
    assert lib.w4_status_string(99) == b"W4_ERR_UNKNOWN"


def test_validation_happens_before_any_cuda_call():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    st = lib.w4_gemv(null, 0, null, null, null, 0, 1, 128, 8, 0, 0, null)
    assert st == _lib.W4_ERR_INVALID_ARG
    assert b"null pointer" in lib.w4_last_error()
    fake = ctypes.c_void_p(4096)
    st = lib.w4_gemv(fake, 0, fake, fake, fake, 0, 1, 100, 8, 0, 0, null)  # K % 128
    assert st == _lib.W4_ERR_INVALID_ARG
    st = lib.w4_gemv(fake, 0, fake, fake, fake, 0, 17, 128, 8, 0, 0, null)  # M > 16
    assert st == _lib.W4_ERR_INVALID_ARG
    st = lib.w4_gemv(fake, 3, fake, fake, fake, 0, 1, 128, 8, 0, 0, null)  # dtype
    assert st == _lib.W4_ERR_INVALID_ARG
    odd = ctypes.c_void_p(4098)
    st = lib.w4_gemv(odd, 0, fake, fake, fake, 0, 1, 128, 8, 0, 0, null)
    assert st == _lib.W4_ERR_ALIGNMENT
    st = lib.w4_pack(fake, 0, fake, fake, 100, 8, 128, null)
    assert st == _lib.W4_ERR_INVALID_ARG
    st = lib.w4_dequant(fake, fake, fake, 0, 128, 12, null)  # N % 8
    assert st == _lib.W4_ERR_INVALID_ARG


def test_tuner_validation_happens_before_any_cuda_call():
    lib = _lib.load()
    cfg = _lib.GemvConfig()
    us = ctypes.c_float(0)
    for args in ((0, 128, 8, 0, 0, 0, 0),      # M < 1
                 (17, 128, 8, 0, 0, 0, 0),     # M > 16
                 (1, 100, 8, 0, 0, 0, 0),      # K % 128
                 (1, 128, 12, 0, 0, 0, 0),     # N % 8
                 (1, 128, 8, 2, 0, 0, 0),      # x dtype
                 (1, 256, 8, 0, 0, 3, 0),      # split_k > K / 128
                 (1, 128, 8, 0, 0, 0, 6)):     # num_warps
        assert lib.w4_gemv_tune(*args, ctypes.byref(cfg), ctypes.byref(us)) == \
            _lib.W4_ERR_INVALID_ARG, args
    assert lib.w4_gemv_tune(1, 128, 8, 0, 0, 0, 0, None, None) == _lib.W4_ERR_INVALID_ARG


def test_decode_step_validation_happens_before_any_cuda_call():
    import ctypes

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.w4_decode_step(None, None, 0, None) == _lib.W4_ERR_INVALID_ARG
    assert lib.w4_decode_step_scratch_bytes(None, ctypes.byref(n)) == _lib.W4_ERR_INVALID_ARG
    d = _lib.DecodeModel(layers=2, hidden=512, intermediate=1024, heads=4, kv_heads=2,
                         head_dim=128, vocab=1000, max_seq=64, eps=1e-6)
    for name, _ in _lib.DecodeModel._fields_[9:]:
        setattr(d, name, 1 << 20)  # fake, aligned device addresses (never dereferenced)
    d.logits = None
    d.head_dim = 64
    assert lib.w4_decode_step(ctypes.byref(d), 1 << 20, 1 << 20, None) == _lib.W4_ERR_UNSUPPORTED
    d.head_dim = 128
    d.heads = 3  # heads * head_dim != hidden
    assert lib.w4_decode_step(ctypes.byref(d), 1 << 20, 1 << 20, None) == _lib.W4_ERR_INVALID_ARG
    d.heads = 4
    d.embed = None
    assert lib.w4_decode_step(ctypes.byref(d), 1 << 20, 1 << 20, None) == _lib.W4_ERR_INVALID_ARG
    d.embed = (1 << 20) + 8
    assert lib.w4_decode_step(ctypes.byref(d), 1 << 20, 1 << 20, None) == _lib.W4_ERR_ALIGNMENT


def test_check_maps_status_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.W4_ERR_INVALID_ARG, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.W4_ERR_ALIGNMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.W4_ERR_UNSUPPORTED, "x")
    with pytest.raises(_lib.W4Error):
        _lib.check(_lib.W4_ERR_CUDA, "x")
    _lib.check(_lib.W4_OK, "x")


def test_no_cpu_fallback_in_product_path():
    """The product package never imports the oracle."""
    import pathlib

    pkg = pathlib.Path(_lib.__file__).parent
    for py in pkg.rglob("*.py"):
        src = py.read_text()
        assert "oracle" not in re.sub(r"#.*", "", src).replace("the oracle", ""), py


def test_lm_head_entry_points_reject_unbuilt_hidden_sizes_before_any_cuda_call():
    """Both argmax entry points accept only the built hidden sizes, and say so
    before any device work (the static one before it looks up its array)."""
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)
    ws_bytes = int(lib.w4_lm_head_workspace_bytes())
    for hidden in (100, 768, 1280, 1792, 4096):
        st = lib.w4_lm_head_argmax_static(fake, fake, 1e-6, fake, 1000, hidden, None, fake,
                                          fake, 0, None)
        assert st == _lib.W4_ERR_UNSUPPORTED, hidden
        st = lib.w4_lm_head_argmax(fake, fake, 1e-6, fake, 1000, hidden, None, fake, fake, fake,
                                   ws_bytes, 0, None)
        assert st == _lib.W4_ERR_UNSUPPORTED, hidden
    assert lib.w4_lm_head_argmax_static(fake, fake, 1e-6, fake, 0, 1536, None, fake, fake, 0,
                                        None) == _lib.W4_ERR_INVALID_ARG


def test_plan_validation_happens_before_any_cuda_call():
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)
    plan = ctypes.c_void_p()
    assert lib.w4_gemv_plan_create(fake, fake, 1, 128, 8, 0, 0, None, None) == \
        _lib.W4_ERR_INVALID_ARG
    for args in ((0, 128, 8, 0, 0),     # M < 1
                 (17, 128, 8, 0, 0),    # M > 16
                 (1, 100, 8, 0, 0),     # K % 128
                 (1, 128, 12, 0, 0),    # N % 8
                 (1, 128, 8, 2, 0)):    # x dtype
        assert lib.w4_gemv_plan_create(fake, fake, *args, None, ctypes.byref(plan)) == \
            _lib.W4_ERR_INVALID_ARG, args
        assert plan.value is None
    odd = ctypes.c_void_p((1 << 20) + 4)
    assert lib.w4_gemv_plan_create(odd, fake, 1, 128, 8, 0, 0, None, ctypes.byref(plan)) == \
        _lib.W4_ERR_ALIGNMENT
    assert lib.w4_gemv_plan_launch(None, fake, fake, None) == _lib.W4_ERR_INVALID_ARG
    assert lib.w4_gemv_plan_launch_host(None, None, fake, fake, None, None) == \
        _lib.W4_ERR_INVALID_ARG
    assert lib.w4_gemv_plan_destroy(None) == _lib.W4_OK
