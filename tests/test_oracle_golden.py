"""The CPU oracle (oracle/oracle.cpp, f32, reference op order) against the float64
numpy restatement's fixtures (tests/golden/c1_small.npz, tests/golden/make_golden.py).

Parity with the reference itself is unpinned (the reference is TypeScript + WGSL with
no CPU path and no golden vectors); these fixtures pin the oracle."""
import numpy as np
import pytest

import oracle
from conftest import max_abs_rel


@pytest.fixture(scope="module")
def run(golden):
    o = oracle.Oracle(n_layers=2, max_seq=64, with_fm=True)
    toks, a0, na = golden["tokens"], int(golden["audio_start"]), int(golden["audio_count"])
    voice, noise = golden["voice"], golden["noise"]
    for i, t in enumerate(toks):
        o.backbone_step(int(t), embed=voice[i - a0] if a0 <= i < a0 + na else None)
    kick = o.backbone_step(24, debug=True, lm_head=True)
    f0 = o.fm_forward(noise[0])
    emb = o.multi_codebook_embed(f0["semantic_code"], f0["acoustic_codes"])
    s1 = o.backbone_step(0, embed=emb, debug=True)
    f1 = o.fm_forward(noise[1])
    yield {"kick": kick, "f0": f0, "s1": s1, "f1": f1}
    o.close()


def test_backbone_layers_match_f64(run, golden):
    for i in range(golden["kick_debug"].shape[0]):
        assert max_abs_rel(run["kick"]["debug"][i], golden["kick_debug"][i]) < 1e-5
        assert max_abs_rel(run["s1"]["debug"][i], golden["f1_debug"][i]) < 1e-5


def test_lm_head_argmax(run, golden):
    assert run["kick"]["argmax"] == int(golden["kick_argmax"])


@pytest.mark.parametrize("f", ["f0", "f1"])
def test_fm_matches_f64(run, golden, f):
    r = run[f]
    assert max_abs_rel(r["semantic_logits"], golden[f + "_semantic_logits"]) < 1e-5
    assert max_abs_rel(r["x_final"], golden[f + "_x_final"]) < 1e-5
    assert r["semantic_code"] == int(golden[f + "_semantic_code"])
    assert np.array_equal(r["acoustic_codes"], golden[f + "_acoustic_codes"])


def test_masked_argmax_rule():
    x = np.zeros(8320, np.float32)
    x[0] = 100.0          # masked (EMPTY_AUDIO)
    x[9000 % 8320] = 0.0
    x[8200] = 50.0        # masked (>= 8194)
    x[5] = 3.0
    x[7] = 3.0            # tie: lowest index wins
    assert oracle.masked_argmax(x) == 5


def test_shader_argmax_rule():
    x = np.full(1000, -5.0, np.float32)
    x[300] = 2.0
    x[44] = 2.0           # tie across lanes: the reference's tree keeps the lower lane
    assert oracle.argmax_shader(x) == 44
