"""The C ABI on a machine without a GPU: the library loads, exports every
function include/*.h declares, and fails loudly (negative status, message)
instead of falling back to anything when no device is present."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT, load_pkg_module

HEADERS = [os.path.join(ROOT, "include", h) for h in ("engine_cuda.h", "ec_transformer.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(ec_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def eng():
    e = load_pkg_module("engine")
    if not os.path.exists(e.LIB_PATH):
        pytest.skip("libengine_cuda.so not built")
    return e


def test_exports_every_declared_symbol(eng):
    lib = C.CDLL(eng.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the binding covers the same list
    assert sorted(eng.EXPORTS) == names


def test_default_config_is_reference_defaults(eng):
    c = eng.ModelConfig()
    assert eng.lib().ec_config_default(C.byref(c)) == 0
    # config.h:67-79 and ops_lsh.h:33-38
    assert (c.sparse_k, c.window, c.sparse_blocks_k) == (64, 128, 64)
    assert (c.lsh_tables, c.lsh_bits, c.lsh_unit, c.lsh_max_units, c.lsh_radius) == \
        (1, 16, 64, 4096, 4)
    assert c.use_paged_kv == 1


def test_config_struct_layout_matches_header(eng):
    """ec_config_default writes exactly sizeof(ec_model_config) bytes: the
    ctypes mirror has the header's size (no byte past it is touched) and
    the fields the header appended last (attention_mode, wait_limit) default
    to 0."""
    n = C.sizeof(eng.ModelConfig)
    buf = (C.c_uint8 * (n + 64))(*([0xAB] * (n + 64)))
    assert eng.lib().ec_config_default(C.cast(buf, C.POINTER(eng.ModelConfig))) == 0
    assert bytes(buf[n:]) == b"\xab" * 64
    c = eng.ModelConfig.from_buffer(buf)
    assert c.attention_mode == 0 and c.wait_limit == 0 and c.max_batch == 1
    assert bytes(buf[n - 4:n]) == b"\x00" * 4


def test_argument_errors_without_device(eng):
    L = eng.lib()
    assert L.ec_create(None, 0, None) == eng.EC_ERR_ARG
    c = eng.ModelConfig()
    L.ec_config_default(C.byref(c))
    c.head_dim = 96 + 256  # unsupported
    h = C.c_void_p()
    assert L.ec_create(C.byref(c), 0, C.byref(h)) == eng.EC_ERR_UNSUPPORTED
    assert L.ec_last_error()
    assert L.ec_op_gemv(0, None, None, None, None, 4, 32, None) == eng.EC_ERR_ARG
    # sampling: missing buffers, non-positive temperature / top_p / penalty,
    # a history without its lengths -- rejected before any device work
    assert L.ec_op_sample_top_p(None, 10, 1, None, None, 0, 0.7, 0.9, 1.2, 1, None, None,
                                None) == eng.EC_ERR_ARG
    fake = C.c_void_p(16)  # never dereferenced: the arguments fail first
    assert L.ec_op_sample_top_p(fake, 10, 1, None, None, 0, 0.0, 0.9, 1.2, 1, fake, fake,
                                None) == eng.EC_ERR_ARG
    assert L.ec_op_sample_top_p(fake, 10, 1, None, None, 0, 0.7, 0.0, 1.2, 1, fake, fake,
                                None) == eng.EC_ERR_ARG
    assert L.ec_op_sample_top_p(fake, 10, 1, fake, None, 4, 0.7, 0.9, 1.2, 1, fake, fake,
                                None) == eng.EC_ERR_ARG
    assert L.ec_op_sample_temperature(fake, 0, 1, 0.7, fake, fake, None) == eng.EC_ERR_ARG
    # context bias: no context / a table without arrays
    assert L.ec_set_context_bias(None, None, None, None, 4) == eng.EC_ERR_ARG


def test_no_device_fails_loudly(eng):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    c = eng.ModelConfig()
    eng.lib().ec_config_default(C.byref(c))
    c.n_layers, c.vocab_size, c.dim, c.hidden_dim = 1, 64, 64, 64
    c.n_heads, c.n_kv_heads, c.head_dim, c.seq_len = 1, 1, 64, 64
    h = C.c_void_p()
    rc = eng.lib().ec_create(C.byref(c), 0, C.byref(h))
    assert rc == eng.EC_ERR_CUDA and not h.value
    assert eng.lib().ec_last_error()
