"""Writes reference_kat.json: the hand-checked values that the reference's
own tests assert, transcribed from their source text (the reference has no
golden data files).  Each entry cites the test it comes from.

Run: python tests/golden/make_kat.py
"""
import json
import os

KAT = {
    "scalar_ops.gemm_2x2_identity": {
        "source": "tests/scalar_ops.rs:3-10",
        "a": [1.0, 2.0, 3.0, 4.0], "identity": [1.0, 0.0, 0.0, 1.0],
        "expected": [1.0, 2.0, 3.0, 4.0],
    },
    "scalar_ops.softmax_rows_sums_to_one": {
        "source": "tests/scalar_ops.rs:12-20",
        "x": [1.0, 2.0, 3.0, 0.0, 0.0, 0.0],
    },
    "scalar_ops.layerscale": {
        "source": "tests/scalar_ops.rs:40-47",
        "x": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "gamma": [10.0, -1.0, 0.5],
        "expected": [10.0, -2.0, 1.5, 40.0, -5.0, 3.0],
    },
    "cuda.gemm_bias_scale": {
        "source": "src/cuda.rs:1399-1417",
        "left": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "right": [7.0, 8.0, 9.0, 10.0, 11.0, 12.0],
        "product": [58.0, 64.0, 139.0, 154.0],
        "bias": [1.0, -4.0], "gamma": [0.5, 2.0],
        "epilogue": [29.5, 120.0, 70.0, 300.0],
    },
    "cuda.prepared_linear_chain": {
        "source": "src/cuda.rs:1433-1447",
        "left": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "rows": 2,
        "first": {"k": 3, "n": 2, "weight": [7.0, 8.0, 9.0, 10.0, 11.0, 12.0], "bias": [1.0, -4.0],
                  "scale": [0.5, 2.0]},
        "second": {"k": 2, "n": 1, "weight": [2.0, -1.0], "bias": [3.0]},
        "expected": [-58.0, -157.0],
    },
    "cuda.add": {
        "source": "src/cuda.rs:1375-1381",
        "a": [1.0, -2.0, 3.5], "b": [0.5, 2.0, -1.0], "expected": [1.5, 0.0, 2.5],
    },
    "cuda.patchify_nchw": {
        "source": "src/cuda.rs:1576-1590",
        "channels": 3, "height": 4, "width": 4, "patch": 2,
        "image": "arange(48)",
        "expected": [0.0, 1.0, 4.0, 5.0, 16.0, 17.0, 20.0, 21.0, 32.0, 33.0, 36.0, 37.0, 2.0, 3.0, 6.0,
                     7.0, 18.0, 19.0, 22.0, 23.0, 34.0, 35.0, 38.0, 39.0, 8.0, 9.0, 12.0, 13.0, 24.0,
                     25.0, 28.0, 29.0, 40.0, 41.0, 44.0, 45.0, 10.0, 11.0, 14.0, 15.0, 26.0, 27.0, 30.0,
                     31.0, 42.0, 43.0, 46.0, 47.0],
    },
    "cuda.prepend_cls_add_pos": {
        "source": "src/cuda.rs:1592-1605",
        "patches": [10.0, 20.0, 30.0, 40.0], "cls": [1.0, 2.0],
        "position": [0.5, -0.5, 1.0, 2.0, -1.0, 3.0], "tokens": 2, "channels": 2,
        "expected": [1.5, 1.5, 11.0, 22.0, 29.0, 43.0],
    },
    "tolerances": {
        "source": "tests/attention_matches_naive.rs:34-41; src/specialized.rs:2871-2910; "
                  "tests/q8_0_dot_matches_f32.rs:54-60; src/cuda.rs:1613-1648",
        "attention_tiled_vs_naive_abs": 1e-4,
        "flash_vs_serial_mae": 2e-5, "flash_vs_serial_max": 2e-4,
        "q8_0_vs_dequantised_f32": [1e-2, 1e-2],
        "cuda_attention_mae": 5e-5, "cuda_attention_max": 5e-4,
    },
}

if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kat.json")
    with open(out, "w") as f:
        json.dump(KAT, f, indent=1)
    print(out)
