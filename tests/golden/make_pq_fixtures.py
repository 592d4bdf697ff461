"""Generate tests/golden/pq_fixtures.json with the reference's own format tools.

1. Q4K packing: sha256 of tools/quant.py quantize_pack(4, w) for seeded matrices.
2. Whole files: a synthetic tiny Qwen3.5 checkpoint is written in the Hugging Face layout
   (config.json + model.safetensors, F32) and converted by the reference's tools/convert.py
   with --quant q4k; the sha256 of the resulting .pq is recorded. nibblemac_b200.pq must write
   the same bytes from the same values without the reference (tests/test_pq_format.py).

Needs the reference checkout (its tools/ are imported and run); runs only where one is
mounted. The fixture it writes is what the tests read.

    python tests/golden/make_pq_fixtures.py /path/to/reference
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from nibblemac_b200 import pq  # noqa: E402

QUANT_CASES = [  # (rows, cols, seed, std, outliers)
    (8, 256, 1, 0.05, False), (16, 512, 2, 0.05, True), (64, 1024, 3, 0.02, False),
    (256, 2048, 4, 0.02, True), (4, 3584, 5, 1.0, False)]


def quant_matrix(rows: int, cols: int, seed: int, std: float, outliers: bool) -> np.ndarray:
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
    if outliers:
        w[:, ::37] *= np.float32(6.0)
        w[1] += np.float32(0.02)
        w[2, :256] = np.float32(0.5)         # a constant group run
        w[3] = 0.0                           # an all-zero row
    return w


def write_hf_checkpoint(d: pq.Dims, seed: int, out: Path) -> None:
    """The synthetic model as a Hugging Face checkpoint (values as nibblemac_b200.pq draws
    them): zero-centred norms store w = multiplier - 1, conv1d is [C, 1, K]."""
    zc = ("input_layernorm.weight", "post_attention_layernorm.weight", "q_norm.weight",
          "k_norm.weight")
    zc_exact = ("norm.weight", "mtp.norm.weight", "mtp.pre_fc_norm_embedding.weight",
                "mtp.pre_fc_norm_hidden.weight")
    header, blobs, off = {}, [], 0
    for name, kind, shape in pq.tensor_specs(d):
        v = pq.tensor_values(name, kind, shape, seed, 0.02)
        if name.endswith(zc) or name in zc_exact:
            v = (v - np.float32(1.0)).astype(np.float32)
        if kind == "conv":
            v = v.reshape(shape[0], 1, shape[1])
        data = np.ascontiguousarray(v, dtype="<f4").tobytes()
        header[pq.hf_name(name)] = {"dtype": "F32", "shape": list(v.shape),
                                    "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    hjson = json.dumps(header).encode()
    with (out / "model.safetensors").open("wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for b in blobs:
            f.write(b)
    layer_types = ["full_attention" if (d.full_mask >> i) & 1 else "linear_attention"
                   for i in range(d.n_layers)]
    cfg = {"text_config": {
        "hidden_size": d.hidden, "num_hidden_layers": d.n_layers, "vocab_size": d.vocab,
        "intermediate_size": d.ffn, "num_attention_heads": d.n_heads,
        "num_key_value_heads": d.n_kv_heads, "head_dim": d.head_dim,
        "rope_parameters": {"rope_theta": d.rope_theta,
                            "partial_rotary_factor": d.rot_dim / d.head_dim},
        "linear_num_key_heads": d.lin_k_heads, "linear_num_value_heads": d.lin_v_heads,
        "linear_key_head_dim": d.lin_k_dim, "linear_value_head_dim": d.lin_v_dim,
        "linear_conv_kernel_dim": d.conv_k, "layer_types": layer_types,
        "eos_token_id": d.eos_id, "tie_word_embeddings": True, "rms_norm_eps": d.rms_eps}}
    (out / "config.json").write_text(json.dumps(cfg))


def main() -> None:
    # the reference checkout: argument, $NB_REFERENCE, else `reference` beside this repository
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else
               os.environ.get("NB_REFERENCE", Path(__file__).resolve().parents[3] / "reference"))
    sys.path.insert(0, str(ref / "tools"))
    import quant  # the reference's quantiser

    fixture: dict = {"about": "made by the reference's tools/quant.py and tools/convert.py",
                     "quant": [], "models": []}
    for rows, cols, seed, std, outl in QUANT_CASES:
        packed = quant.quantize_pack(4, quant_matrix(rows, cols, seed, std, outl))[0]
        fixture["quant"].append({"rows": rows, "cols": cols, "seed": seed, "std": std,
                                 "outliers": outl,
                                 "sha256": hashlib.sha256(packed).hexdigest()})
    for preset, seed in (("tiny", 1), ("small", 2)):
        d = pq.PRESETS[preset]
        with tempfile.TemporaryDirectory() as td:
            tdp = Path(td)
            write_hf_checkpoint(d, seed, tdp)
            out = tdp / "m.pq"
            subprocess.run([sys.executable, str(ref / "tools" / "convert.py"), str(tdp),
                            str(out), "--quant", "q4k"], check=True, capture_output=True)
            fixture["models"].append({"preset": preset, "seed": seed,
                                      "sha256": pq.sha256_file(out)})
    path = Path(__file__).with_name("pq_fixtures.json")
    path.write_text(json.dumps(fixture, indent=1) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
