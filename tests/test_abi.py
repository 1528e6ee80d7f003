"""The C-ABI library loads without a GPU and exports every symbol the header declares."""
import ctypes
import re
import subprocess

import pytest


def test_library_exports_header_symbols(vx):
    lib = vx.load_library()
    syms = vx.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), s


def test_nm_matches_header(vx):
    out = subprocess.run(["nm", "-D", "--defined-only", vx.library_path()], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (vx_[a-z_0-9]+)\b", out))
    assert set(vx.header_symbols()) <= exported


def test_default_config_matches_reference(vx):
    c = vx.default_config()
    # defaultConfig (src/types.ts:70-97)
    assert (c.dim, c.n_layers, c.head_dim, c.hidden_dim, c.n_heads, c.n_kv_heads, c.vocab_size) == \
        (3072, 26, 128, 9216, 32, 8, 131072)
    assert c.rope_theta == 1e6 and abs(c.norm_eps - 1e-5) < 1e-12
    assert (c.fm_n_layers, c.fm_nfe, c.fm_n_acoustic, c.fm_semantic_vocab) == (3, 8, 36, 8320)
    assert abs(c.fm_cfg_alpha - 1.2) < 1e-6 and c.max_seq_len == 4096


def test_bad_config_rejected_without_gpu(vx):
    c = vx.default_config()
    c.tp_size = 3
    h = ctypes.c_void_p()
    rc = vx.load_library().vx_create(ctypes.byref(c), ctypes.byref(h))
    assert rc == -1
    assert b"tp_size" in vx.load_library().vx_last_error(h)
    vx.load_library().vx_destroy(h)


def test_engine_without_gpu_fails_loudly(vx):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}})
    with pytest.raises(vx.VoxtralError):
        e.init()
    assert not e.isReady
    with pytest.raises(vx.VoxtralError, match="not initialized"):
        e.generate([1, 2], 0, 0, None, 1)


def test_node_binding_covers_header(vx):
    """The committed Node binding (webgpu-voxtral_b200/node/voxtral_b200.ts, untested here:
    no Node in this container) binds every function the header declares, with the
    header's name."""
    import os
    ts = open(os.path.join(os.path.dirname(vx.library_path()), "node", "voxtral_b200.ts")).read()
    bound = set(re.findall(r"lib\.func\('[^(']*?\b(vx_[a-z_0-9]+)\(", ts))
    assert set(vx.header_symbols()) <= bound, set(vx.header_symbols()) - bound
