"""Generate tests/golden/*.npz from the reference itself (oracle/_ref, built from its sources).

    make -C oracle ref && python tests/golden/make_golden.py

Inputs are regenerated from seeds by tests/golden/cases.py (numpy PCG64), so the fixtures store
only the reference's outputs plus a SHA-256 of every input, which the tests re-check to catch
any drift in input generation. Outputs come from the reference's own functions:
qms_quantize_q8, qms_vec_dot_q8, qms_vec_dot_f32, qms_dequant_row and moe() with --trace.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402
from oracle import Reference  # noqa: E402


def main():
    ref = Reference()
    ref.set_threads(4)
    out = {"ref_variant": np.array(ref.variant)}

    # qms_quantize_q8 (src/kernels.c:34-53)
    for name, x in cases.quant_cases().items():
        out[f"quant/{name}/sha"] = np.array(cases.sha(x))
        out[f"quant/{name}/q8"] = ref.quantize_q8(x).view(np.uint8)

    # qms_vec_dot_q8 / qms_vec_dot_f32 (src/kernels.c:82-219)
    for name, (typ, n, w, x) in cases.dot_cases().items():
        xq = ref.quantize_q8(x).reshape(len(w), -1)
        out[f"dot/{name}/sha"] = np.array(cases.sha(w, x))
        out[f"dot/{name}/got"] = np.array([ref.vec_dot_q8(typ, w[i], xq[i], n) for i in range(len(w))],
                                          np.float32)
    for name, (w, x) in cases.f32_cases().items():
        out[f"f32/{name}/sha"] = np.array(cases.sha(w, x))
        out[f"f32/{name}/got"] = np.array([ref.vec_dot_f32(w[i], x) for i in range(len(w))], np.float32)

    # qms_dequant_row (src/quant.c:109-121), cross-checked bit-exactly against gguf-py's
    # dequantisers as the reference's tools/test_deq.py:19-47 does
    import gguf
    for name, (typ, n, blob) in cases.deq_cases().items():
        got = ref.dequant_row(typ, blob, n)
        g = gguf.quants.dequantize(blob, gguf.GGMLQuantizationType(typ)).reshape(-1).astype(np.float32)
        assert np.array_equal(got.view(np.uint32), g.view(np.uint32)), f"reference != gguf-py on {name}"
        out[f"deq/{name}/sha"] = np.array(cases.sha(blob))
        out[f"deq/{name}/got"] = got

    # moe() (src/model.c:1032-1167), resident integer path, with its --trace records
    for name, (layer, xn) in cases.moe_cases().items():
        o, tr = ref.moe(layer, xn, trace=True)
        out[f"moe/{name}/sha"] = np.array(cases.sha(layer.router, layer.gate, layer.up, layer.down, xn))
        out[f"moe/{name}/out"] = o
        out[f"moe/{name}/trace"] = tr

    path = HERE / "reference_golden.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size / 1e3:.0f} kB, {len(out)} arrays, reference {ref.variant})")


if __name__ == "__main__":
    main()
