"""Generate tests/golden/c2_depth.npz with the C++ oracle (oracle/oracle.cpp) at full depth.

Run from the repository root:  python tests/golden/make_depth_golden.py
(a few minutes of CPU on 8 cores; the output is committed).

Case: configs[1] of the benchmark (C2) at full depth, cut to 16 frames: the 26-layer
backbone with synthetic weights (seed 0), utterance 11 with the C2 prompt (512 text ids
+ 100 voice rows = 617 positions), prefilled token by token as the reference does
(src/engine.ts:2457-2472), then the AUDIO kick and 15 backbone-only frames fed with the
synthetic feedback codes of stream (4, utt) (src/engine.ts:2498-2541 with the codes
injected).  Saved: the final-norm state of every frame (the FM's input), f32 [16][3072].

The oracle itself is pinned at the C1 shape to the float64 restatement
(tests/golden/c1_small.npz); this fixture extends the comparison to 26 layers and a
617-position prompt, where the oracle is too slow to run inside a GPU test.
"""
from __future__ import annotations

import importlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

synth = importlib.import_module("webgpu-voxtral_b200.synth")

UTT, N_TEXT, N_VOICE, N_FRAMES, N_LAYERS = 11, 512, 100, 16, 26


def main(out=os.path.join(ROOT, "tests", "golden", "c2_depth.npz")):
    t0 = time.time()
    o = oracle.Oracle(n_layers=N_LAYERS, max_seq=4096, with_fm=False)
    print(f"weights {time.time() - t0:.1f}s ({oracle.num_threads()} threads)", flush=True)
    toks, a0, na = synth.prompt(UTT, N_TEXT, N_VOICE)
    voice = synth.voice_rows(UTT, N_VOICE)
    codes_in = synth.feedback_codes(UTT, 0, N_FRAMES)
    ref = o.generate(toks, a0, na, voice, N_FRAMES, codes_in=codes_in, want_normed=True)
    o.close()
    np.savez_compressed(out, utt=UTT, n_text=N_TEXT, n_voice=N_VOICE, n_layers=N_LAYERS, positions=len(toks),
                        normed=ref["normed"].astype(np.float32))
    print(f"wrote {out} in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
