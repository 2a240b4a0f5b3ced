"""Writes the layer golden fixtures in this folder: the oracle's exact-f32 layer (quant::dequant
feeding moe_layer_forward, src/moe.rs:360-388) on seeded synthetic inputs.  The inputs are not
stored: they are regenerated from the same seeds by rusty_engine_b200.synth, whose generator is
deterministic (numpy PCG64).  Run from the repository root:

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402
from rusty_engine_b200 import synth  # noqa: E402
from rusty_engine_b200.synth import GGML_Q4_K, GGML_Q5_0, GGML_Q6_K, GGML_Q8_0  # noqa: E402

# name -> (layer builder, tokens, activation seed)
CASES = {
    "c1_t16": (lambda: synth.config_c1(), 16, 5),
    "kq_sigmoid_shared_t12": (lambda: synth.make_layer(512, 256, 8, 2, gate_t=GGML_Q4_K, up_t=GGML_Q4_K,
                                                       down_t=GGML_Q6_K, dlo=0.002, dhi=0.02, seed=11, gate=1,
                                                       shared=True, name="kq-sig-sh"), 12, 6),
    "q5_0_q8_0_t7": (lambda: synth.make_layer(256, 512, 4, 3, gate_t=GGML_Q5_0, up_t=GGML_Q5_0, down_t=GGML_Q8_0,
                                              dlo=0.0015, dhi=0.006, seed=12, name="q5q8"), 7, 7),
}


def compute(name):
    build, T, seed = CASES[name]
    lw = build()
    x = synth.activations(T, lw.H, seed=seed)
    out, ids, w, logits = O.moe_layer_q_exact(x, lw, threads=1)
    return lw, x, out, ids, w, logits


def main():
    for name in CASES:
        _, _, out, ids, w, logits = compute(name)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out=out, ids=ids, w=w, logits=logits)
        print(name, out.shape)


if __name__ == "__main__":
    main()
