"""Regenerates tests/golden/oracle_config0.json: the CPU oracle's output for
BASELINE config 0 (one token, seed 0, layer 0), pinned so that any change to
the oracle's arithmetic is visible.  Run from the repo root:
    python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def main():
    seed, layer, tok0, T = 0, 0, 0, 1
    L = O.OracleLayer.synth(seed, layer)
    x = O.synth_hidden(seed, tok0, T)
    r = O.block(L, x, threads=0)
    g = {
        "what": "oracle qfo_block on BASELINE config 0: seed 0, layer 0, token 0",
        "seed": seed, "layer": layer, "tok0": tok0, "T": T,
        "x_sha256": hashlib.sha256(x.tobytes()).hexdigest(),
        "idx": r["idx"].tolist(),
        "w": r["w"].tolist(),
        "coef": float(r["coef"][0]),
        "logits_sha256": hashlib.sha256(r["logits"].tobytes()).hexdigest(),
        "out_sha256": hashlib.sha256(r["out"].tobytes()).hexdigest(),
        "out_head": r["out"][0, :8].tolist(),
    }
    with open(os.path.join(HERE, "oracle_config0.json"), "w") as f:
        json.dump(g, f, indent=1)
    print(json.dumps(g)[:300])


if __name__ == "__main__":
    main()
