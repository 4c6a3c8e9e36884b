"""Generate tests/golden/sampler_golden.npz from the reference's own sample() (src/chat.c:36-69,
built into oracle/_ref/libqms_ref_sample.so from the reference's sources):

    make -C oracle ref && python tests/golden/make_sampler_golden.py

Inputs are regenerated from seeds by cases.sampler_cases(); the fixture keeps, per case, a SHA-256
of the logits and the reference's token and generator state after each of two draws in a row.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402
from oracle import RefSampler  # noqa: E402


def main():
    ref = RefSampler()
    out = {}
    for name, (l, temp, top_p, top_k, seed) in cases.sampler_cases().items():
        st, toks, states = seed, [], []
        for _ in range(2):
            t, st = ref.sample(l, temp, top_p, top_k, st)
            toks.append(t)
            states.append(st)
        out[f"{name}/sha"] = np.array(cases.sha(l))
        out[f"{name}/tokens"] = np.array(toks, np.int64)
        out[f"{name}/states"] = np.array(states, np.uint64)
    path = HERE / "sampler_golden.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({len(out) // 3} cases)")


if __name__ == "__main__":
    main()
