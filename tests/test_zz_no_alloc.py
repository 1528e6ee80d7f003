"""vx_lm_head_argmax_noalloc: the LM-head argmax for callers that cannot allocate.

Callers such as a real-time audio callback (where cudaMalloc may synchronise the device
and block) or a host framework that owns all device memory cannot create a vx_handle.
They pass their own device buffers to this entry point, which allocates nothing: its
scratch is a static device array.  This test gives it device buffers allocated by the
test itself (the caller's memory) and checks it, through the C ABI, against the
handle-based path (vx_backbone_step with argmax_out) on two calls in a row, within the
suite's tolerance (indices exact, the maximum logit within 2e-2 relative).

Kept in its own file so that pytest collects it last; it is self-contained and runs
alone in a fresh process as well as after the other tests."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 2e-2


def test_lm_head_argmax_noalloc_matches_handle_path(vx, synth):
    import torch

    L = vx.load_library()
    fn = L.vx_lm_head_argmax_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]

    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 16,
                            "enableFM": False})
    eng.init()
    eng.loadRandomWeights(0)
    toks, a0, na = synth.prompt(9, 6, 2)
    eng.reset()
    eng.prefill(toks, a0, na, synth.voice_rows(9, 2))
    normed, want_idx = eng.backboneStep(24, lmHead=True)          # handle-based path (engine scratch)
    emb = eng.readTensor("mm_audio_embeddings.tok_embeddings.weight")
    eng.destroy()

    rows, dim = 131072, 3072
    dev = torch.device("cuda", 0)
    w = torch.from_numpy(emb.view(np.int16).reshape(rows, dim)).to(dev)     # caller-owned device memory
    x = torch.from_numpy(normed).to(dev)
    idx = torch.full((1,), -1, dtype=torch.int32, device=dev)
    val = torch.zeros(1, dtype=torch.float32, device=dev)
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream(dev)
    ref_val = float(emb[want_idx * dim:(want_idx + 1) * dim].astype(np.float64) @ normed.astype(np.float64))
    for _ in range(2):                                               # two calls in a row share the scratch
        idx.fill_(-1)
        rc = fn(w.data_ptr(), x.data_ptr(), rows, dim, idx.data_ptr(), val.data_ptr(), stream.cuda_stream, err, 256)
        assert rc == 0, err.value
        torch.cuda.synchronize()
        assert int(idx.item()) == want_idx
        assert abs(float(val.item()) - ref_val) <= TOL * abs(ref_val)

    rc = fn(w.data_ptr(), x.data_ptr(), 2_097_153, dim, idx.data_ptr(), None, stream.cuda_stream, err, 256)
    assert rc == -4 and b"rows" in err.value                      # beyond the scratch's maximum


def _noalloc_fn(vx):
    fn = vx.load_library().vx_lm_head_argmax_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return fn


@pytest.mark.parametrize("rows,dim", [(1000, 264), (200, 3072), (1, 8), (257, 16384)])
def test_lm_head_argmax_noalloc_small_and_ragged(vx, rows, dim):
    """Ragged last CTA (rows not a multiple of 256), a single-CTA grid, K loops that stop
    early (dim not a multiple of 256) and the tie rule: a copy of the maximum row placed
    at a lower index must win.  Checked against a float64 numpy argmax."""
    import torch

    fn = _noalloc_fn(vx)
    rng = np.random.default_rng(rows + dim)
    w = (rng.standard_normal((rows, dim)) * 0.02).astype(np.float16)
    x = rng.standard_normal(dim).astype(np.float32)
    dots = w.astype(np.float64) @ x.astype(np.float64)
    top = int(np.argmax(dots))
    if rows > 1 and top > 0:
        dup = top // 2
        w[dup] = w[top]                       # identical products: the lower index wins
        dots = w.astype(np.float64) @ x.astype(np.float64)
    want = int(np.argmax(dots))               # numpy returns the first maximum
    second = np.partition(dots, -2)[-2] if rows > 1 else -np.inf
    dev = torch.device("cuda", 0)
    wd = torch.from_numpy(w.view(np.int16)).to(dev)
    xd = torch.from_numpy(x).to(dev)
    idx = torch.full((1,), -2, dtype=torch.int32, device=dev)
    val = torch.zeros(1, dtype=torch.float32, device=dev)
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream(dev)
    for _ in range(2):
        idx.fill_(-2)
        rc = fn(wd.data_ptr(), xd.data_ptr(), rows, dim, idx.data_ptr(), val.data_ptr(), stream.cuda_stream, err, 256)
        assert rc == 0, err.value
        torch.cuda.synchronize()
        got = int(idx.item())
        if dots[want] - second > 1e-4 * abs(dots[want]) or second == dots[want]:
            assert got == want, (got, want)
        assert abs(float(val.item()) - dots[want]) <= TOL * abs(dots[want])


def test_lm_head_argmax_noalloc_all_nan(vx):
    import torch

    fn = _noalloc_fn(vx)
    dev = torch.device("cuda", 0)
    wd = torch.ones((300, 64), dtype=torch.float16, device=dev).view(torch.int16)
    xd = torch.full((64,), float("nan"), dtype=torch.float32, device=dev)
    idx = torch.zeros(1, dtype=torch.int32, device=dev)
    val = torch.zeros(1, dtype=torch.float32, device=dev)
    err = ctypes.create_string_buffer(256)
    rc = fn(wd.data_ptr(), xd.data_ptr(), 300, 64, idx.data_ptr(), val.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream, err, 256)
    assert rc == 0, err.value
    torch.cuda.synchronize()
    assert int(idx.item()) == -1 and np.isnan(float(val.item()))
