"""Generate golden vectors from the reference's own CPU code.

The reference's ``spark_mlx_llm/conversion.py`` needs only NumPy, so it can be
imported here (by file path, without ``mlx``) to produce known outputs of its
bf16 rounding (``bf16``, :154-160), affine packing (``_packed``, :429-433) and
quantizer (``_rows``, :551-608). The outputs are written to
``conversion_vectors.npz`` next to this script; the tests compare the oracle's
restatement against them bit for bit.

Run (where the reference tree is present):
    python tests/golden/make_golden.py --reference PATH
The GPU box does not have the reference; it uses the committed ``.npz``.
"""

import argparse
import importlib.util
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_conversion(reference):
    path = Path(reference) / "spark_mlx_llm" / "conversion.py"
    spec = importlib.util.spec_from_file_location("_ref_conversion", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def bf16_words(values):
    """Truncation-free bf16 encoding used only to build *inputs* (exact values)."""
    words = np.asarray(values, dtype="<f4").view(np.uint32)
    return ((words + 0x7FFF + ((words >> 16) & 1)) >> 16).astype("<u2")


def edge_floats():
    ties = np.array(
        [
            1.0 + 2.0**-8,  # exact tie, even neighbour below
            1.0 + 3 * 2.0**-8,  # exact tie, even neighbour above
            -(1.0 + 2.0**-8),
            1.0 + 2.0**-8 + 2.0**-20,  # just above a tie
            1.0 + 2.0**-8 - 2.0**-20,  # just below a tie
        ],
        dtype=np.float32,
    )
    specials = np.array(
        [0.0, -0.0, 1e-40, -1e-40, 1.17549435e-38, 3.0e38, -3.0e38, 65504.0, 1e-8],
        dtype=np.float32,
    )
    return np.concatenate([ties, specials])


def write_tensor(directory, name, data, dtype, shape):
    path = Path(directory) / name
    raw = np.ascontiguousarray(data).tobytes()
    path.write_bytes(raw)
    return {"path": path, "offset": 0, "dtype": dtype, "shape": list(shape), "bytes": len(raw)}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference project tree")
    args = parser.parse_args()
    conv = load_conversion(args.reference)
    rng = np.random.default_rng(20260101)
    out = {}

    # 1. bf16 rounding (conversion.py:154-160).
    values = np.concatenate(
        [
            rng.standard_normal(4096).astype(np.float32),
            (rng.standard_normal(1024) * 1e-3).astype(np.float32),
            (rng.standard_normal(1024) * 1e4).astype(np.float32),
            edge_floats(),
        ]
    )
    encoded, decoded = conv.bf16(values)
    out["bf16_in"] = values
    out["bf16_bits"] = encoded.astype(np.uint16)
    out["bf16_decoded"] = decoded.astype(np.float32)

    # 2. affine packing (conversion.py:429-433).
    for bits in (2, 4, 8):
        codes = rng.integers(0, 1 << bits, size=(7, 64), dtype=np.uint32)
        out[f"pack{bits}_codes"] = codes
        out[f"pack{bits}_words"] = conv._packed(codes, bits)

    # 3. the reference quantizer (conversion.py:551-608).
    rows, k = 12, 128
    w = (rng.standard_normal((rows, k)) * 0.02).astype(np.float32)
    w[0] = 0.0  # all-zero row/groups -> scale 1
    w[1] = np.abs(w[1]) + 0.01  # all-positive -> lower clamps to 0
    w[2] = -np.abs(w[2]) - 0.01  # all-negative -> upper clamps to 0
    w[3, :32] = 0.5  # constant group
    w[4] *= 100.0  # wide range
    w_bits = bf16_words(w)
    out["rows_w_bf16_bits"] = w_bits
    with tempfile.TemporaryDirectory() as tmp:
        src = write_tensor(tmp, "w.bin", w_bits, "BF16", (rows, k))
        cases = [
            ("w4", "model.layers.0.mlp.gate_proj", {"kind": "bf16-int4", "bits": 4}),
            ("w8", "model.layers.0.self_attn.out_proj", {"kind": "bf16-int8", "bits": 8}),
            ("w8f32", "lm_head", {"kind": "bf16-int8", "bits": 8}),
        ]
        for tag, module, scheme in cases:
            scheme = dict(scheme, shape=[rows, k])
            result, _ = conv._rows(module, scheme, {module + ".weight": src}, 0, rows)
            out[f"rows_{tag}_weight"] = np.frombuffer(result["weight"], "<u4").reshape(rows, -1)
            coef = "<f4" if module == "lm_head" else "<u2"
            out[f"rows_{tag}_scales"] = np.frombuffer(result["scales"], coef).reshape(rows, -1)
            out[f"rows_{tag}_biases"] = np.frombuffer(result["biases"], coef).reshape(rows, -1)

        # channel-int8: existing int8 codes with a per-row BF16 weight_scale.
        codes = rng.integers(-127, 128, size=(rows, k), dtype=np.int8)
        scale = (np.abs(rng.standard_normal((rows, 1))) * 1e-3 + 1e-4).astype(np.float32)
        scale_bits = bf16_words(scale)
        module = "model.layers.1.self_attn.out_proj"
        tensors = {
            module + ".weight": write_tensor(tmp, "q.bin", codes, "I8", (rows, k)),
            module + ".weight_scale": write_tensor(tmp, "s.bin", scale_bits, "BF16", (rows, 1)),
        }
        scheme = {"kind": "channel-int8", "bits": 8, "shape": [rows, k]}
        result, _ = conv._rows(module, scheme, tensors, 0, rows)
        out["chan_codes"] = codes
        out["chan_scale_bf16_bits"] = scale_bits
        out["rows_chan_weight"] = np.frombuffer(result["weight"], "<u4").reshape(rows, -1)
        out["rows_chan_scales"] = np.frombuffer(result["scales"], "<u2").reshape(rows, -1)
        out["rows_chan_biases"] = np.frombuffer(result["biases"], "<u2").reshape(rows, -1)

    np.savez_compressed(HERE / "conversion_vectors.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'conversion_vectors.npz'}")


if __name__ == "__main__":
    main()
