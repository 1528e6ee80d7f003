"""Generate tests/golden/c1_small.npz with the float64 numpy restatement.

Run from the repository root:  python tests/golden/make_golden.py
(about three minutes of CPU; the output is committed).

Case: the C1 model shape (2 backbone layers, full width, 3 FM layers), synthetic
weights (seed 0), utterance 0 with 4 text tokens and 2 voice rows:
  prefill 11 tokens -> AUDIO kick (debug tensors of debugBackboneLayerByLayer and the
  greedy LM-head argmax of backboneStepAndRead) -> frame 0 FM with noise[0] ->
  frame 1 backbone step on the multi-codebook embedding of frame 0's codes (debug
  tensors) -> frame 1 FM with noise[1].
"""
from __future__ import annotations

import importlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import numpy_ref  # noqa: E402

synth = importlib.import_module("webgpu-voxtral_b200.synth")

N_TEXT, N_VOICE, UTT = 4, 2, 0


def main(out=os.path.join(ROOT, "tests", "golden", "c1_small.npz")):
    t0 = time.time()
    m = numpy_ref.RefModel(n_layers=2, with_fm=True, lm_head=True)
    print(f"weights {time.time() - t0:.1f}s", flush=True)
    toks, a0, na = synth.prompt(UTT, N_TEXT, N_VOICE)
    voice = synth.voice_rows(UTT, N_VOICE)
    noise = synth.fm_noise(UTT, 0, 2)
    for i, t in enumerate(toks):
        m.step(int(t), embed=voice[i - a0] if a0 <= i < a0 + na else None)
    kick = m.step(24, debug=True)
    f0 = m.fm_forward(kick["normed"], noise[0])
    emb = m.multi_codebook_embed(f0["semantic_code"], f0["acoustic_codes"])
    s1 = m.step(0, embed=emb, debug=True)
    f1 = m.fm_forward(s1["normed"], noise[1])
    np.savez_compressed(
        out,
        tokens=toks, audio_start=a0, audio_count=na, voice=voice, noise=noise,
        kick_debug=kick["debug"].astype(np.float32), kick_argmax=kick["argmax"],
        f0_semantic_logits=f0["semantic_logits"].astype(np.float32), f0_x_final=f0["x_final"].astype(np.float32),
        f0_acoustic_codes=f0["acoustic_codes"], f0_semantic_code=f0["semantic_code"],
        f1_debug=s1["debug"].astype(np.float32),
        f1_semantic_logits=f1["semantic_logits"].astype(np.float32), f1_x_final=f1["x_final"].astype(np.float32),
        f1_acoustic_codes=f1["acoustic_codes"], f1_semantic_code=f1["semantic_code"],
    )
    print(f"wrote {out} in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
