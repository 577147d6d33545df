"""Generate tests/golden/kquant_gguf.npz by executing the REFERENCE's own GGUF
code (ef_deepseek_mmap.py, read from a reference checkout given by
--reference or the EF_REFERENCE environment variable):

* ``dequant_q2_k_fast`` / ``dequant_q3_k_fast`` / ``dequant_q4_k_fast``
  (ef_deepseek_mmap.py:330-378, 655-773) on seeded K-quant blocks -- typical
  super-block scales plus blocks whose fp16 scales are arbitrary finite bit
  patterns (subnormal, negative, overflowing on output);
* the scalar ``dequant_q2_k`` (ef_deepseek_mmap.py:282-327) on four blocks;
* ``tensor_byte_size`` (ef_deepseek_mmap.py:188-197) over every block type;
* ``parse_split_gguf`` and ``ExpertMmapLoader`` (ef_deepseek_mmap.py:248-275,
  383-593) on a two-file DeepSeek-style model written by
  ``expertflow_b200.gguf.write_gguf``: parsed tensor infos, each expert's raw
  byte range and a digest of each expert's dequantised matrices.

Run:  python tests/golden/make_gguf_golden.py --reference <reference checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import os
import sys
import tempfile
from contextlib import redirect_stdout

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from expertflow_b200 import gguf as G  # noqa: E402

OUT = os.path.join(HERE, "kquant_gguf.npz")
N_TYPICAL, N_WILD = 40, 8
MODEL = {"E": 4, "hidden": 512, "inter": 256, "layers": {1: (G.GGML_TYPE_Q2_K, G.GGML_TYPE_Q3_K, G.GGML_TYPE_Q4_K),
                                                         2: (G.GGML_TYPE_Q4_K, G.GGML_TYPE_Q2_K, G.GGML_TYPE_Q3_K)},
         "seed": 77}


def wild_blocks(dtype: int, n: int, rng: np.random.Generator) -> bytes:
    """Blocks whose fp16 scale fields are random finite bit patterns."""
    per, bb = G.GGML_BLOCK_SIZES[dtype]
    raw = np.frombuffer(G.random_kquant_blocks(dtype, n, rng), np.uint8).reshape(n, bb).copy()
    fields = {G.GGML_TYPE_Q2_K: (80, 82), G.GGML_TYPE_Q3_K: (108,), G.GGML_TYPE_Q4_K: (0, 2)}[dtype]
    for off in fields:
        bits = rng.integers(0, 0x7C00, size=n).astype(np.uint16) | (rng.integers(0, 2, size=n).astype(np.uint16) << 15)
        raw[:, off:off + 2] = bits.view(np.uint8).reshape(n, 2)
    return raw.tobytes()


def model_tensors():
    rng = np.random.default_rng(MODEL["seed"])
    E, H, I = MODEL["E"], MODEL["hidden"], MODEL["inter"]
    files = [{}, {}]
    for fi, (layer, types) in enumerate(sorted(MODEL["layers"].items())):
        for proj, dt in zip(("gate", "up", "down"), types):
            cols, rows = (H, I) if proj != "down" else (I, H)
            shape = (cols, rows, E)
            nb = cols * rows * E // 256
            files[fi][f"blk.{layer}.ffn_{proj}_exps.weight"] = (shape, dt, G.random_kquant_blocks(dt, nb, rng))
        files[fi][f"blk.{layer}.attn_norm.weight"] = ((H,), G.GGML_TYPE_F32,
                                                      rng.standard_normal(H).astype(np.float32).tobytes())
    meta = [{"general.architecture": "deepseek2", "deepseek2.expert_count": E, "deepseek2.block_count": 3,
             "deepseek2.leading_dense_block_count": 1, "deepseek2.rope.freq_base": 10000.0,
             "tokenizer.ggml.tokens": ["a", "b", "c"], "general.flag": True},
            {"general.architecture": "deepseek2", "split.no": 1}]
    return files, meta, [32, 64]


def write_model(d: str):
    files, meta, align = model_tensors()
    paths = []
    for i, (t, m, a) in enumerate(zip(files, meta, align)):
        p = os.path.join(d, f"model-{i + 1:05d}-of-00002.gguf")
        G.write_gguf(p, t, m, alignment=a)
        paths.append(p)
    return paths


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EF_REFERENCE"),
                    required="EF_REFERENCE" not in os.environ,
                    help="reference checkout to import (default: $EF_REFERENCE)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import ef_deepseek_mmap as R

    out = {}
    fast = {G.GGML_TYPE_Q2_K: R.dequant_q2_k_fast, G.GGML_TYPE_Q3_K: R.dequant_q3_k_fast,
            G.GGML_TYPE_Q4_K: R.dequant_q4_k_fast}
    for k, dt in enumerate(G.KQUANT_TYPES):
        rng = np.random.default_rng(100 + k)
        blocks = G.random_kquant_blocks(dt, N_TYPICAL, rng) + wild_blocks(dt, N_WILD, rng)
        n = N_TYPICAL + N_WILD
        with np.errstate(over="ignore", invalid="ignore"):
            y = fast[dt](np.frombuffer(blocks, np.uint8), (n * 256,))
        out[f"blocks_{dt}"] = np.frombuffer(blocks, np.uint8)
        out[f"dequant_{dt}"] = y.view(np.uint16)
    raw = out[f"blocks_{G.GGML_TYPE_Q2_K}"][:4 * 84]
    out["q2k_scalar"] = R.dequant_q2_k(raw, (1024,)).view(np.uint16)
    sizes = []
    for dt in sorted(R.GGML_BLOCK_SIZES):
        for shape in ((256,), (1024,), (257,), (512, 64), (256, 1024, 8), (7168, 2048, 4)):
            try:
                sizes.append((dt, *shape, *([0] * (3 - len(shape))), len(shape), R.tensor_byte_size(shape, dt)))
            except ValueError:
                pass
    out["byte_sizes"] = np.array(sizes, np.int64)

    with tempfile.TemporaryDirectory() as d:
        paths = write_model(d)
        out["model_file_sha"] = np.array([sha(open(p, "rb").read()) for p in paths])
        with redirect_stdout(io.StringIO()):
            infos, tensors, meta = R.parse_split_gguf(d)
            loader = R.ExpertMmapLoader(d, verbose=False)
        parsed = {"data_offsets": [i.data_offset for i in infos], "alignments": [i.alignment for i in infos],
                  "versions": [i.version for i in infos], "metadata": meta,
                  "tensors": {n: [list(t.shape), t.dtype, t.offset, t.file_idx, t.total_bytes]
                              for n, t in sorted(tensors.items())}}
        out["parsed_json"] = np.array(json.dumps(parsed, sort_keys=True))
        rows = []
        for layer in sorted(MODEL["layers"]):
            for e in range(MODEL["E"]):
                g, u, dn = loader.load_expert_dequantized(layer, e)
                for proj, mat in zip(("gate", "up", "down"), (g, u, dn)):
                    rawb, dt, shape = loader.load_expert_raw(layer, e, proj)
                    rows.append([layer, e, proj, dt, json.dumps(list(shape)), sha(rawb), sha(mat.view(np.uint16))])
                if layer == 1 and e == 2:
                    out["expert_1_2_down"] = dn.reshape(-1).view(np.uint16)[:8192]
        out["experts"] = np.array(rows)
        loader.close()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
