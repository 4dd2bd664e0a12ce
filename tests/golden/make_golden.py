"""Regenerates the committed golden fixtures in tests/golden/.

Run in a container that has gguf-py 0.19.0 (the version the reference pins in
scripts/envs/qwen3-tts/uv.lock:291-293) and, optionally, the reference tree:

    python tests/golden/make_golden.py [--reference /path/to/synthesize.cpp]

What it writes, and which reference artefact each fixture pins:

* q8_pack_fixtures.json -- Q8_0 packing (quantize_row_q8_0_ref) of
  - the (i+1)/7 tensor from tests/synthesize_quantize_test.cpp:33-41,55
    (decoder.post.weight [7,32,1] packed as one 224-wide row, :264-278),
  - hand-made edge rows (zeros, ties at .5, negative ties, fp16-overflowing
    scales, fp16-subnormal scales, fp32 subnormals, one-hot rows),
  all produced by gguf-py's Q8_0 quantizer (gguf/quants.py:378-394), which
  states bit-exactness with ggml-quants.c.
* q8_seeded_digests.json -- SHA-256 digests of the seeded inputs of
  BASELINE config 1 (W = 0.02*N(0,1) seed 0 [3072x1024], x = N(0,1) seed 1
  [1024]) as drawn by the reference's own NormalRandomStream
  (src/random-stream.cpp, compiled into oracle/_ref) when available, and of
  their gguf-py packing; plus the full packed x.
* vits_q8_cases.json -- the two Q8_0 conv-as-matmul cases of
  tests/vits_conv_test.cpp:293-313 restated as MUL_MAT inputs, with the
  reference's expected outputs and its bound of 0.5 (:106-110).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402


def gguf_pack(x: np.ndarray) -> np.ndarray:
    from gguf import GGMLQuantizationType, quants

    return quants.quantize(np.ascontiguousarray(x, dtype=np.float32), GGMLQuantizationType.Q8_0)


def edge_rows() -> dict[str, np.ndarray]:
    rows: dict[str, np.ndarray] = {}
    rows["zeros"] = np.zeros(32, np.float32)
    rows["neg_zeros"] = -np.zeros(32, np.float32)
    # amax 127 -> d = 1, id = 1: x*id lands exactly on .5 ties
    t = np.arange(32, dtype=np.float32) - 15.5
    t[0] = 127.0
    rows["ties_half"] = t
    rows["ties_half_neg"] = -t
    # amax 254 -> d = 2: x/2 ties at odd integers
    rows["ties_odd"] = np.concatenate([[254.0], np.arange(-61, 1, 2, dtype=np.float32)]).astype(np.float32)
    rows["one_hot"] = np.eye(32, dtype=np.float32)[5] * 3.25
    rows["one_hot_neg"] = -np.eye(32, dtype=np.float32)[31] * 1e-3
    rows["fp16_overflow_scale"] = np.linspace(-3e38, 3e38, 32, dtype=np.float32)
    rows["fp16_subnormal_scale"] = np.linspace(-1e-6, 2e-6, 32, dtype=np.float32)
    rows["fp32_tiny"] = np.linspace(-1e-30, 1e-30, 32, dtype=np.float32)
    rows["constant"] = np.full(32, 0.1, np.float32)
    rows["ramp_1_7"] = (np.arange(64, dtype=np.float32) + 1) / np.float32(7)
    rng = np.random.default_rng(1234)
    rows["wide_dynamic"] = (rng.standard_normal(96) * np.exp(rng.uniform(-20, 20, 96))).astype(np.float32)
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SYNTH_REFERENCE", ""),
                    help="reference tree (default: $SYNTH_REFERENCE; the RNG pin is skipped without one)")
    args = ap.parse_args()

    # ---- packing fixtures (gguf-py is the oracle's pin)
    pack = {"generator": "gguf-py 0.19.0 gguf.quants.quantize(x, Q8_0)", "cases": {}}
    seven = (np.arange(224, dtype=np.float32) + 1) / np.float32(7)
    pack["cases"]["synthesize_quantize_test_i_plus_1_over_7"] = {
        "source": "tests/synthesize_quantize_test.cpp:33-41,55,264-278",
        "k": 224,
        "x_f32_hex": seven.tobytes().hex(),
        "q8_0_hex": gguf_pack(seven.reshape(1, -1)).tobytes().hex(),
        "probe": {"index": 100, "expected": float(101 / 7), "bound": 0.2},
    }
    for name, row in edge_rows().items():
        pack["cases"][name] = {
            "source": "hand-made edge row",
            "k": int(row.size),
            "x_f32_hex": row.astype(np.float32).tobytes().hex(),
            "q8_0_hex": gguf_pack(row.reshape(1, -1)).tobytes().hex(),
        }
    with open(os.path.join(HERE, "q8_pack_fixtures.json"), "w") as f:
        json.dump(pack, f, indent=1)

    # ---- seeded config-1 digests
    if args.reference and os.path.isdir(os.path.join(args.reference, "src")):
        O.build(args.reference)
    ref = O.ref_lib()

    def draw(seed: int, n: int) -> np.ndarray:
        if ref is not None:
            out = np.empty(n, np.float32)
            ref.ref_normal_fill(seed, out.ctypes.data, n)
            return out
        return O.normal(seed, n)

    w = (np.float32(0.02) * draw(0, 3072 * 1024)).astype(np.float32).reshape(3072, 1024)
    x = draw(1, 1024).reshape(1, 1024)
    wq = gguf_pack(w)
    xq = gguf_pack(x)
    seeded = {
        "rng": "reference src/random-stream.cpp via oracle/_ref" if ref is not None else "oracle restatement",
        "config1": {
            "w_shape": [3072, 1024], "w_seed": 0, "w_scale": 0.02,
            "x_shape": [1, 1024], "x_seed": 1,
            "w_f32_sha256": hashlib.sha256(w.tobytes()).hexdigest(),
            "x_f32_sha256": hashlib.sha256(x.tobytes()).hexdigest(),
            "w_q8_0_sha256": hashlib.sha256(wq.tobytes()).hexdigest(),
            "x_q8_0_hex": xq.tobytes().hex(),
            "first_normals_seed0": [float(v) for v in draw(0, 8)],
        },
    }
    with open(os.path.join(HERE, "q8_seeded_digests.json"), "w") as f:
        json.dump(seeded, f, indent=1)

    # ---- vits conv-as-matmul cases (loose reference pins)
    cases = []
    # case A: 1x1 conv, in 32, out 2; kernel rows of 1.0 and -0.5; bias {0.25,-0.75};
    # input frame f channel c = f + c + 1
    wA = np.concatenate([np.ones(32, np.float32), np.full(32, -0.5, np.float32)]).reshape(2, 32)
    xA = np.array([[f + c + 1 for c in range(32)] for f in range(3)], np.float32)
    expA = []
    for f in range(3):
        s = float(xA[f].sum())
        expA.append([s + 0.25, -0.5 * s - 0.75])
    cases.append({"source": "tests/vits_conv_test.cpp:293-309", "k": 32, "w_f32": wA.ravel().tolist(),
                  "n": 2, "x_f32": xA.ravel().tolist(), "m": 3, "bias": [0.25, -0.75],
                  "expected": expA, "bound": 0.5})
    # case B: kernel 3, in 32, out 1, all ones, 4 frames of ones, padding 1, bias 0.5.
    # im2col rows: frame t reads input frames t-1, t, t+1 (zero outside) for each of 32 channels.
    wB = np.ones((1, 96), np.float32)
    xB = np.zeros((4, 96), np.float32)
    for t in range(4):
        for tap in range(3):
            src = t - 1 + tap
            if 0 <= src < 4:
                xB[t, tap * 32:(tap + 1) * 32] = 1.0
    cases.append({"source": "tests/vits_conv_test.cpp:310-313", "k": 96, "w_f32": wB.ravel().tolist(),
                  "n": 1, "x_f32": xB.ravel().tolist(), "m": 4, "bias": [0.5],
                  "expected": [[64.5], [96.5], [96.5], [64.5]], "bound": 0.5})
    with open(os.path.join(HERE, "vits_q8_cases.json"), "w") as f:
        json.dump({"cases": cases}, f, indent=1)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
