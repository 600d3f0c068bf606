"""Regenerates the committed golden fixtures from the reference checkout.

    python tests/golden/make_golden.py <reference checkout>

attention_sync_oracle.npz re-packs the reference's own known-answer vectors
(docs/verification/attention-sync/oracle/{debug.json,tensors.bin}, written by
apps/inspect_main.cpp:61-101): the tiny config, 9 input ids, targets, loss mask,
the weighted-NLL loss, logits [9, 264], and for every parameter its weight, its
gradient and its value after one AdamW update (lr 1e-3). Nothing else is derived.
"""
import json
import os
import sys

import numpy as np


def main(ref):
    src = os.path.join(ref, "docs", "verification", "attention-sync", "oracle")
    with open(os.path.join(src, "debug.json")) as f:
        meta = json.load(f)
    blob = open(os.path.join(src, "tensors.bin"), "rb").read()
    out = {}
    for t in meta["tensors"]:
        a = np.frombuffer(blob, np.float32, t["nbytes"] // 4, t["offset"]).reshape(t["shape"])
        out["t:" + t["name"]] = a.copy()
    out["input"] = np.array([int(x) for x in meta["input"].split(",")], np.uint16)
    out["targets"] = np.array([int(x) for x in meta["targets"].split(",")], np.uint16)
    out["mask"] = np.array([float(x) for x in meta["mask"].split(",")], np.float32)
    out["loss"] = np.array(meta["loss"], np.float64)
    out["learning_rate"] = np.array(meta["learning_rate"], np.float32)
    opt = meta["optimizer"]
    out["optimizer"] = np.array([opt["beta1"], opt["beta2"], opt["epsilon"], opt["weight_decay"],
                                 opt["clip_norm"]], np.float32)
    out["config"] = np.array(json.dumps(meta["config"]))
    out["param_names"] = np.array([p["name"] for p in meta["parameters"]])
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "attention_sync_oracle.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    main(sys.argv[1])
