"""Failure detection without a GPU fault: a bounded device wait made to expire.

Under tensor parallelism the persistent decode kernel waits for every peer's all-reduce
words.  A rank that dies leaves its peers waiting; each wait is bounded and ends in
VX_E_DEVICE instead of a hung GPU.  This test makes that happen on ONE GPU: a tp_size 2
handle in "tp_loopback" mode has every peer receive buffer pointing at its own memory, so
rank 1's words never arrive (a flag that nothing sets).  With a short wait_limit the
decode returns VX_E_DEVICE naming the peer wait, and afterwards the handle and the CUDA
context stay usable.  No second kernel, no peer memory, no fault is involved."""
import numpy as np
import pytest

import oracle
from conftest import max_abs_rel

pytestmark = pytest.mark.gpu
VX_E_DEVICE = -7


def test_lost_peer_wait_expires_and_handle_stays_usable(vx, synth):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 16,
                          "enableFM": False, "enableCodec": False, "tpSize": 2, "tpRank": 0})
    e.init()
    try:
        e.loadRandomWeights(0)
        e.set_option("wait_limit", 1 << 16)   # polls: milliseconds instead of seconds
        e.set_option("tp_loopback", 1)
        e.fill_kv(100, seed=1)
        with pytest.raises(vx.VoxtralError) as ei:
            e.decode(2, with_fm=False)
            e.synchronize()
        assert ei.value.code == VX_E_DEVICE
        assert "peer" in str(ei.value)
        # the handle stays usable: kernels launch and complete, state can be read
        e.fill_kv(50, seed=2)
        e.synchronize()
        assert e.position() == 50
        assert e.read_normed(0, 1).shape == (1, 3072)
    finally:
        e.destroy()
    # the CUDA context stays usable: a tp_size 1 engine decodes and matches the oracle
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 16,
                          "enableFM": False, "enableCodec": False})
    e.init()
    try:
        e.loadRandomWeights(0)
        e.set_streams(noise_seed=3, codes_seed=4, utt=7)
        e.fill_kv(100, seed=1)
        e.decode(2, with_fm=False)
        got = e.read_normed(0, 2)
    finally:
        e.destroy()
    o = oracle.Oracle(n_layers=2, max_seq=256, with_fm=False)
    o.fill_kv(100, seed=1)
    ref0 = o.backbone_step(24)["normed"]
    c = synth.feedback_codes(7, 0, 1)[0]
    ref1 = o.backbone_step(embed=o.multi_codebook_embed(int(c[0]), c[1:]))["normed"]
    o.close()
    assert max_abs_rel(got[0], ref0) < 2e-2
    assert max_abs_rel(got[1], ref1) < 2e-2


def test_options_are_validated(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 1}}, "maxSeqLen": 64, "maxFrames": 8,
                          "enableFM": False, "enableCodec": False})
    e.init()
    try:
        with pytest.raises(vx.VoxtralError, match="unknown option"):
            e.set_option("no_such_option", 1)
        with pytest.raises(vx.VoxtralError, match="l2_prefetch_tiles"):
            e.set_option("l2_prefetch_tiles", 99)
        with pytest.raises(vx.VoxtralError, match="tp_loopback needs"):
            e.set_option("tp_loopback", 1)
        e.set_option("l2_prefetch_tiles", 0)
        e.set_option("persistent_decode", 0)
        e.set_option("persistent_decode", 1)
    finally:
        e.destroy()
