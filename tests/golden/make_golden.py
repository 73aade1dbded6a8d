"""Make the golden fixtures in tests/golden/ from the reference's committed test data (run once, where the
tabicl-anywhere repository is available; the outputs are committed and the GPU box never needs the reference):

    python tests/golden/make_golden.py /path/to/tabicl-anywhere

* tiny-clf.tirs / tiny-reg.tirs: the reference's tiny random TabICL checkpoints (tests/data/tiny-{clf,reg}.ckpt,
  made by its tools/make_tiny.py) as weight bundles: every tensor of the state dict as float32 plus
  config.json, the layout its tools/export_weights.py writes.
* tiny-raw-icl.tirs: the reference's golden dump tests/data/tiny-raw.tirs (PyTorch TabICL's own numbers for the
  tiny classifier) without its plain-attention logits: the normalised training and test rows and training labels,
  training and test row representations, the in-context keys/values of every layer ([heads][rows][head width]) and
  the logits; and for the column and row stages the column stage's cached keys/values of every block ([columns]
  [heads][inducing points][head width], the class-token columns first) and the training and test rows' tokens after
  the column stage.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
import importlib.util  # noqa: E402

spec = importlib.util.spec_from_file_location("tirs", os.path.join(HERE, "..", "..", "tabicl-anywhere_b200", "tirs.py"))
tirs = importlib.util.module_from_spec(spec)
spec.loader.exec_module(tirs)


def weights(ckpt, out):
    ck = torch.load(ckpt, map_location="cpu", weights_only=True)
    t = {k: v.numpy().astype(np.float32) for k, v in ck["state_dict"].items()}
    t["config.json"] = np.frombuffer(json.dumps(ck["config"]).encode(), dtype=np.uint8)
    tirs.write(out, t)
    print(out, len(t), "tensors")


def main(ref):
    data = os.path.join(ref, "tests", "data")
    weights(os.path.join(data, "tiny-clf.ckpt"), os.path.join(HERE, "tiny-clf.tirs"))
    weights(os.path.join(data, "tiny-reg.ckpt"), os.path.join(HERE, "tiny-reg.tirs"))
    raw = tirs.Bundle(os.path.join(data, "tiny-raw.tirs"))
    keep = ["train_rep", "y_train", "test_rep", "logits", "x_test", "test_emb", "x_train", "train_emb"]
    keep += [n for n in raw.names() if n.startswith(("icl_k", "icl_v", "col_k", "col_v"))]
    out = os.path.join(HERE, "tiny-raw-icl.tirs")
    tirs.write(out, {n: np.array(raw[n]) for n in keep})
    print(out, keep)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <checkout of tabicl-anywhere>")
    main(sys.argv[1])
