"""Host-side logic of the VoxtralEngine mirror (no GPU)."""
import numpy as np


def test_sample_top_p_restricts_to_nucleus(vx):
    rng = np.random.default_rng(0)
    logits = np.full(100, -10.0)
    logits[[3, 7]] = [5.0, 4.9]
    seen = {vx.sample_top_p(logits, 0.9, 0.8, rng) for _ in range(200)}
    assert seen <= {3, 7} and seen == {3, 7}


def test_sample_top_p_masked_never_chosen(vx):
    rng = np.random.default_rng(1)
    logits = rng.normal(size=8320)
    logits[0] = -np.inf
    logits[8194:] = -np.inf
    for _ in range(100):
        c = vx.sample_top_p(logits, 0.9, 0.8, rng)
        assert 1 <= c < 8194


def test_options_map_to_config(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}, "fm": {"nfe": 8}}, "maxSeqLen": 1024,
                          "maxSlots": 3})
    assert e.config.n_layers == 2 and e.config.max_seq_len == 1024 and e.config.max_slots == 3
    assert e.config.fm_nfe == 8
    assert not e.isReady


def test_tts_result_shape(vx):
    r = vx.TTSResult(semanticCodes=[5], acousticCodes=[[2] * 36], audio=np.zeros(0, np.float32),
                     stats={"framesGenerated": 1})
    assert r.stats["framesGenerated"] == 1 and r.audio.size == 0
