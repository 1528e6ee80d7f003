"""The persistent decode kernel's hand-off forms compute the same values.

`early_kv_pair` (each CTA's first K / V pair copied during the QKV phase, the current
position's row patched in shared memory afterwards) changes only when data moves, not the
arithmetic: both settings must give bit-identical final-norm states, under either form of
`residual_handoff`.  The two `residual_handoff` forms (the residual handed to the next
phase as tagged words, with q and the current K / V row reaching the attention phase as
tagged words; or added in place behind grid barriers) sum the final norm's squares in
different orders, so they agree to rounding.  Positions are chosen so that the current
row lies in the first pair of its split (crossing a page boundary) and in a later pair of
a split of three pages; every state is also checked against the CPU oracle."""
import itertools

import numpy as np
import pytest

import oracle
from conftest import max_abs_rel

pytestmark = pytest.mark.gpu

FRAMES = 3


def _decode_states(vx, pos, residual_handoff, early_kv_pair):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 1536, "maxFrames": 16,
                          "enableFM": False, "enableCodec": False})
    e.init()
    try:
        e.loadRandomWeights(0)
        e.set_option("residual_handoff", residual_handoff)
        e.set_option("early_kv_pair", early_kv_pair)
        e.set_streams(noise_seed=3, codes_seed=4, utt=7)
        e.fill_kv(pos, seed=1)
        e.decode(FRAMES, with_fm=False)
        return e.read_normed(0, FRAMES)
    finally:
        e.destroy()


# 126: frames at positions 126-128 cross from page 1 into page 2 (one pair per split);
# 1300: 21 pages in 7 splits of 3 pages, so position 1300's page is the second pair of
# the last split.
@pytest.mark.parametrize("pos", [126, 1300])
def test_handoff_forms_agree(vx, synth, pos):
    states = {combo: _decode_states(vx, pos, *combo) for combo in itertools.product((0, 1), (0, 1))}
    for r in (0, 1):
        assert np.array_equal(states[(r, 0)], states[(r, 1)]), f"residual_handoff {r}: early_kv_pair changes the state"
    assert max_abs_rel(states[(0, 1)], states[(1, 1)]) < 1e-5
    o = oracle.Oracle(n_layers=2, max_seq=1536, with_fm=False)
    o.fill_kv(pos, seed=1)
    refs = [o.backbone_step(24)["normed"]]
    codes = synth.feedback_codes(7, 0, FRAMES - 1)
    for c in codes:
        refs.append(o.backbone_step(embed=o.multi_codebook_embed(int(c[0]), c[1:]))["normed"])
    o.close()
    for combo, got in states.items():
        for f in range(FRAMES):
            assert max_abs_rel(got[f], refs[f]) < 2e-2, f"residual_handoff, early_kv_pair = {combo}, frame {f}"


def test_early_kv_pair_option_is_validated(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 1}}, "maxSeqLen": 64, "maxFrames": 8,
                          "enableFM": False, "enableCodec": False})
    e.init()
    try:
        with pytest.raises(vx.VoxtralError, match="early_kv_pair"):
            e.set_option("early_kv_pair", 2)
        e.set_option("early_kv_pair", 0)
        e.set_option("early_kv_pair", 1)
    finally:
        e.destroy()
