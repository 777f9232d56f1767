"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/argus_b200.h declares (no compute calls are made here)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "argus_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(argus_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header_symbols():
    from argus_b200 import _lib
    assert os.path.exists(_lib.LIB_PATH), "build the library first (python -m argus_b200.build)"
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert L.argus_version() >= 100


def test_python_binding_covers_header():
    from argus_b200 import _lib, attention, paged, sharding
    from argus_b200.core import jl
    declared = set(declared_symbols())
    bound = (set(_lib.SIGNATURES) | set(attention.BOUND_SYMBOLS) | set(paged.BOUND_SYMBOLS) | set(jl.BOUND_SYMBOLS)
             | set(sharding.BOUND_SYMBOLS)
             | {"argus_status_string", "argus_last_error", "argus_version"})
    assert declared <= bound, sorted(declared - bound)


def test_status_strings():
    from argus_b200 import _lib
    assert _lib.status_string(0) == "ok"
    assert "misaligned" in _lib.status_string(_lib.ERR_MISALIGNED)


def test_decode_attention_refuses_bad_arguments_before_touching_the_device():
    """argus_decode_attention validates its arguments on the host and returns the status codes
    the header documents (no CUDA call is reached for any of these)."""
    from argus_b200 import _lib
    from argus_b200 import attention as A

    L = A._bind()
    buf = (ctypes.c_uint8 * 4096)()
    base = (ctypes.addressof(buf) + 15) & ~15  # 16-byte aligned host scratch standing in for q / out
    split = (ctypes.c_int32 * 2)(0, 0)
    arenas = (A.ArenaC * A.MAX_ARENAS)()

    def call(shape, chunks=None, q=base, out=base + 1024, arena_ptr=arenas, s_ptr=True):
        return L.argus_decode_attention(ctypes.byref(shape) if s_ptr else None, arena_ptr, chunks, split, q, out,
                                        None, None, None, None)

    def shape(**kw):
        f = dict(batch=1, heads_kv=1, group=4, q_len=1, head_dim=128, n_splits=1, n_arenas=1, n_chunks=0,
                 scale=0.088, flags=0)
        f.update(kw)
        return A.ShapeC(**f)

    assert call(shape(), s_ptr=False) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(), q=None) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(batch=0)) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(n_splits=0)) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(n_arenas=0)) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(n_arenas=A.MAX_ARENAS + 1)) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(n_chunks=1)) == _lib.ERR_INVALID_ARGUMENT  # chunks missing
    assert call(shape(head_dim=48)) == _lib.ERR_UNSUPPORTED
    assert call(shape(batch=256, heads_kv=256)) == _lib.ERR_UNSUPPORTED  # B * H_kv above 65535
    assert call(shape(), q=base + 2) == _lib.ERR_MISALIGNED
    assert call(shape(), out=base + 1026) == _lib.ERR_MISALIGNED
    assert "alignment" in _lib.lib().argus_last_error().decode()


def test_codec_entry_points_refuse_bad_arguments():
    """The quantizers refuse null buffers, head dims that are not a multiple of 8 and sequence
    lengths that are not a multiple of the tier's packing factor (the reference asserts the last,
    core/quantization.py:41,79,183), on the host, before any launch."""
    from argus_b200 import _lib

    L = _lib.lib()  # argument types bound from _lib.SIGNATURES
    buf = (ctypes.c_uint8 * 4096)()
    p = ctypes.addressof(buf)
    for name in ("argus_quant_int8", "argus_quant_fp8sim"):
        fn = getattr(L, name)
        assert fn(None, 4, 64, p, p, None) == _lib.ERR_INVALID_ARGUMENT
        assert fn(p, 4, 64, p, None, None) == _lib.ERR_INVALID_ARGUMENT
        assert fn(p, 4, 60, p, p, None) == _lib.ERR_UNSUPPORTED
    for name, per in (("argus_quant_int4", 2), ("argus_quant_int2", 4), ("argus_quant_1bit", 8)):
        fn = getattr(L, name)
        extra = (p,) if name != "argus_quant_1bit" else ()
        assert fn(p, per + 1, 64, p, p, *extra, None) == _lib.ERR_INVALID_ARGUMENT
        assert "packing factor" in L.argus_last_error().decode()
        assert fn(p, -per, 64, p, p, *extra, None) == _lib.ERR_INVALID_ARGUMENT
        assert fn(p, per, 64, p, None, *extra, None) == _lib.ERR_INVALID_ARGUMENT


def test_wait_timeout_selftest_refuses_bad_arguments():
    from argus_b200 import _lib

    L = _lib.lib()
    g = ctypes.c_int(0)
    assert L.argus_selftest_wait_timeout(0, ctypes.byref(g), None) == _lib.ERR_INVALID_ARGUMENT
    assert L.argus_selftest_wait_timeout((1 << 20) + 1, ctypes.byref(g), None) == _lib.ERR_INVALID_ARGUMENT
    assert L.argus_selftest_wait_timeout(10, None, None) == _lib.ERR_INVALID_ARGUMENT


def test_jl_entry_points_refuse_bad_shapes_before_any_launch():
    """The JL operator layout is R in 128-token pairs and R^T in 64-token chunks, so both JL entry
    points refuse block token counts that are not a multiple of 128, and the attention refuses
    unsupported head dims, block rows, query groups and misaligned blocks, on the host."""
    from argus_b200 import _lib
    from argus_b200.core import jl

    L = jl._jl_bind()
    buf = (ctypes.c_uint8 * 4096)()
    p = ctypes.addressof(buf)
    p16 = (p + 15) & ~15
    assert L.argus_jl_operator_fragments(p16, 192, 64, p16, p16, None) == _lib.ERR_INVALID_ARGUMENT
    assert "multiple of 128" in L.argus_last_error().decode()
    assert L.argus_jl_operator_fragments(p16, 256, 48, p16, p16, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.argus_jl_operator_fragments(None, 256, 64, p16, p16, None) == _lib.ERR_INVALID_ARGUMENT

    def shape(**kw):
        s = dict(batch=1, heads_kv=2, group=4, q_len=1, head_dim=128, block_rows=128, block_tokens=512,
                 n_blocks=3, n_splits=1, n_ctas=0, scale=0.1, reserved=0, bh_stride=3 * 128 * 128,
                 block_stride=128 * 128)
        s.update(kw)
        return jl.JLShapeC(**s)

    def call(s, yk=p16):
        return L.argus_jl_attention(ctypes.byref(s), yk, p16, p16, p16, p16, p16, None, None, p16, None)

    assert call(shape(block_tokens=192)) == _lib.ERR_UNSUPPORTED
    assert "multiple of 128" in L.argus_last_error().decode()
    assert call(shape(head_dim=96)) == _lib.ERR_UNSUPPORTED
    assert call(shape(block_rows=32)) == _lib.ERR_UNSUPPORTED
    assert call(shape(group=9)) == _lib.ERR_UNSUPPORTED
    assert call(shape(n_splits=4)) == _lib.ERR_INVALID_ARGUMENT
    assert call(shape(), yk=p16 + 2) == _lib.ERR_MISALIGNED
