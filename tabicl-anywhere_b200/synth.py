"""Seeded synthetic TabICL v2 weight bundles and in-context inputs for the benchmark configurations.

No checkpoint or dataset is available offline, so the benchmark and the large parity cases use random-init
weights with the published architecture's tensor names and shapes (the layout tabicl-anywhere's Model::load
accepts, src/model.rs:202-272) and seeded synthetic row representations:

* linear and embedding weights and biases ~ N(0, std) (std 0.02 unless given), LayerNorm weights 1 + N(0, std),
  LayerNorm biases N(0, std), rotary frequencies 1 / base^(2i / head width);
* row representations ~ N(0, 1) per coordinate (the row stage ends in a LayerNorm, so its outputs are unit
  scale); training labels uniform over the classes.
"""
import json

import numpy as np

# 1 is the tiny CPU-runnable model, 2-5 the full-size architecture.
ARCH = {
    "tiny": dict(embed_dim=16, col_num_blocks=1, col_nhead=2, col_num_inds=4, row_num_blocks=1, row_nhead=2,
                 row_num_cls=2, icl_num_blocks=2, icl_nhead=2, max_classes=10, num_quantiles=999),
    "full": dict(embed_dim=128, col_num_blocks=3, col_nhead=4, col_num_inds=128, row_num_blocks=3, row_nhead=8,
                 row_num_cls=4, icl_num_blocks=12, icl_nhead=4, max_classes=10, num_quantiles=999),
}


def config(arch="full", regression=False, **over):
    c = dict(ARCH[arch])
    c.update(over)
    if regression:
        c["max_classes"] = 0
    c.update(col_affine=False, col_feature_group="same", col_feature_group_size=3, col_target_aware=True,
             col_ssmax="qassmax-mlp-elementwise", row_rope_base=100000, row_rope_interleaved=False,
             icl_ssmax="qassmax-mlp-elementwise", ff_factor=2, dropout=0.0, activation="gelu", norm_first=True,
             bias_free_ln=False, recompute=False)
    return c


def weights(cfg, seed=0, std=0.02, hid=64):
    """All tensors of a TabICL v2 checkpoint of this configuration, as float32 arrays, plus config.json."""
    rng = np.random.default_rng(seed)
    t = {}

    def lin(name, out, inp, bias=True):
        t[name + ".weight"] = rng.normal(0, std, (out, inp)).astype(np.float32)
        if bias:
            t[name + ".bias"] = rng.normal(0, std, (out,)).astype(np.float32)

    def ln(name, n):
        t[name + ".weight"] = (1 + rng.normal(0, std, (n,))).astype(np.float32)
        t[name + ".bias"] = rng.normal(0, std, (n,)).astype(np.float32)

    def block(p, d, heads, ff, ssmax):
        lin(p + ".linear1", ff, d)
        lin(p + ".linear2", d, ff)
        ln(p + ".norm1", d)
        ln(p + ".norm2", d)
        t[p + ".attn.in_proj_weight"] = rng.normal(0, std, (3 * d, d)).astype(np.float32)
        t[p + ".attn.in_proj_bias"] = rng.normal(0, std, (3 * d,)).astype(np.float32)
        lin(p + ".attn.out_proj", d, d)
        if ssmax:
            s = p + ".attn.ssmax_layer."
            lin(s + "base_mlp.0", hid, 1)
            lin(s + "base_mlp.2", d, hid)
            lin(s + "query_mlp.0", hid, d // heads)
            lin(s + "query_mlp.2", d // heads, hid)

    e, ff = cfg["embed_dim"], cfg["ff_factor"]
    mc = cfg["max_classes"]
    lin("col_embedder.in_linear", e, cfg["col_feature_group_size"])
    for i in range(cfg["col_num_blocks"]):
        p = f"col_embedder.tf_col.blocks.{i}"
        t[p + ".ind_vectors"] = rng.normal(0, std, (cfg["col_num_inds"], e)).astype(np.float32)
        block(p + ".multihead_attn1", e, cfg["col_nhead"], ff * e, True)
        block(p + ".multihead_attn2", e, cfg["col_nhead"], ff * e, False)
    lin("col_embedder.y_encoder", e, mc if mc > 0 else 1)
    t["row_interactor.cls_tokens"] = rng.normal(0, std, (cfg["row_num_cls"], e)).astype(np.float32)
    for i in range(cfg["row_num_blocks"]):
        block(f"row_interactor.tf_row.blocks.{i}", e, cfg["row_nhead"], ff * e, False)
    hd_row = e // cfg["row_nhead"]
    t["row_interactor.tf_row.rope.freqs"] = (1.0 / cfg["row_rope_base"] ** (np.arange(0, hd_row, 2) / hd_row)).astype(np.float32)
    ln("row_interactor.out_ln", e)
    d = e * cfg["row_num_cls"]
    for i in range(cfg["icl_num_blocks"]):
        block(f"icl_predictor.tf_icl.blocks.{i}", d, cfg["icl_nhead"], ff * d, True)
    ln("icl_predictor.ln", d)
    lin("icl_predictor.y_encoder", d, mc if mc > 0 else 1)
    lin("icl_predictor.decoder.0", ff * d, d)
    lin("icl_predictor.decoder.2", mc if mc > 0 else cfg["num_quantiles"], ff * d)
    t["config.json"] = np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8)
    return t


def icl_shape(cfg, hid=64):
    d = cfg["embed_dim"] * cfg["row_num_cls"]
    mc = cfg["max_classes"]
    return dict(d=d, heads=cfg["icl_nhead"], layers=cfg["icl_num_blocks"], ff=cfg["ff_factor"] * d, hid=hid,
                dec_ff=cfg["ff_factor"] * d, outs=mc if mc > 0 else cfg["num_quantiles"], max_classes=mc)


def rows_shape(cfg):
    """The column and row stages' sizes (tcu_rows_shape) of this configuration."""
    e = cfg["embed_dim"]
    return dict(e=e, group=cfg["col_feature_group_size"], inds=cfg["col_num_inds"], cls=cfg["row_num_cls"],
                col_heads=cfg["col_nhead"], row_heads=cfg["row_nhead"], col_blocks=cfg["col_num_blocks"],
                row_blocks=cfg["row_num_blocks"], col_ff=cfg["ff_factor"] * e, row_ff=cfg["ff_factor"] * e)


def features(n, f, seed, missing=0.0):
    """Seeded normalised feature rows [n][f] ~ N(0, 1) (prep standardises columns, src/prep.rs:4), a fraction
    `missing` of the cells -100 (prep's marker for a missing value)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, f)).astype(np.float32)
    if missing:
        x[rng.random((n, f)) < missing] = -100.0
    return x


def col_kv(features, blocks, e, inds, seed, digits=1):
    """A seeded stand-in for a fitted member's column-stage cache (fit.rs:230: [features][digits][blocks][2][e][inds];
    each group's inducing points' keys and values, unit scale)."""
    return np.random.default_rng(seed).standard_normal((features, digits, blocks, 2, e, inds)).astype(np.float32)


def row_reps(n, d, seed):
    """Seeded synthetic row representations [n][d] (unit scale, as the row stage's final LayerNorm leaves them)."""
    return np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)


def labels(n, classes, seed):
    return np.random.default_rng(seed).integers(0, classes, n).astype(np.float32)
