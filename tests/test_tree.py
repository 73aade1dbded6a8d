"""The class tree on the host: fit::Plan (src/fit.rs:151-221) and its stored form, and the oracle's restatement of
the tree step of prediction (src/predict.rs:664-692), each against answers worked out by hand; and the names and sizes
of the tensors a fit fills (fit::raw_entries, src/fit.rs:224-241)."""
import pytest
import numpy as np

from conftest import tcu
import oracle

Plan = tcu.Plan


def _labels(counts):
    return np.concatenate([np.full(c, k, np.float32) for k, c in enumerate(counts)])


def test_plan_of_few_classes_is_one_leaf():
    y = _labels([4, 3, 5])
    p = Plan.new(10, y, 3)
    assert p.bases == [3]
    assert len(p.nodes) == 1 and p.nodes[0].leaf and p.nodes[0].rows is None and p.nodes[0].map == [0, 1, 2]
    assert p.tree(12).tolist() == [1, 12, 3, 0, 1, 2]


def test_plan_of_a_regressor_is_one_leaf():
    p = Plan.new(0, np.zeros(5, np.float32), 999)
    assert p.bases == [999] and p.nodes[0].k == 999 and p.nodes[0].leaf


def test_plan_of_fourteen_classes():
    """14 classes, 10 told apart: 2 digits of base 4 (16 >= 14), a root telling 2 groups of 7 apart, 2 leaves."""
    y = _labels([3] * 14)
    rng = np.random.default_rng(0)
    y = y[rng.permutation(len(y))]
    p = Plan.new(10, y, 14)
    assert p.bases == [4, 4]
    root, a, b = p.nodes
    assert not root.leaf and root.k == 2 and root.map == [1, 2] and root.rows == list(range(42))
    assert a.leaf and a.map == list(range(7)) and b.leaf and b.map == list(range(7, 14))
    # each node's rows are its classes' rows, in order; targets are local (group or class within the leaf)
    assert a.rows == [r for r in range(42) if y[r] < 7] and b.rows == [r for r in range(42) if y[r] >= 7]
    assert np.array_equal(root.y, (y >= 7).astype(np.float32))
    assert np.array_equal(b.y, y[b.rows] - 7)
    assert p.tree(42).tolist() == [0, 42, 2, 1, 2, 1, 21, 7, *range(7), 1, 21, 7, *range(7, 14)]


def test_plan_of_many_classes_is_three_levels():
    """150 classes: 3 digits of base 6; a root over 10 groups of 15, each an inner node over groups of 8 and 7."""
    y = _labels([2] * 150)
    p = Plan.new(10, y, 150)
    assert p.bases == [6, 6, 6]
    assert len(p.nodes) == 31
    root = p.nodes[0]
    assert root.k == 10 and not root.leaf
    for g, child in enumerate(root.map):
        inner = p.nodes[child]
        assert not inner.leaf and inner.k == 2
        lo, hi = (p.nodes[c] for c in inner.map)
        assert lo.map == list(range(15 * g, 15 * g + 8)) and hi.map == list(range(15 * g + 8, 15 * g + 15))
    # nodes come in the order they were grown: a parent before its children
    for i, n in enumerate(p.nodes):
        assert all(c > i for c in ([] if n.leaf else n.map))


def test_plan_uses_the_classes_present():
    """More classes than told apart, but only three of them among the rows: a single leaf over those three."""
    y = np.array([0, 5, 20, 5, 0], np.float32)
    p = Plan.new(10, y, 25)
    assert len(p.nodes) == 1 and p.nodes[0].map == [0, 5, 20]
    assert p.nodes[0].y.tolist() == [0, 1, 2, 1, 0]


def test_tree_scores_known_answer():
    """Root over {node 1: classes 0, 1; node 2: class 2} at even odds; node 1 three to one for class 0."""
    tree = [0, 4, 2, 1, 2, 1, 2, 2, 0, 1, 1, 2, 1, 2]
    f = np.float32
    s0 = np.zeros((1, 2), f)
    s1 = np.array([[0.9 * np.log(3.0), 0.0]], f)
    s2 = np.array([[5.0]], f)
    got = oracle.tree_scores([s0, s1, s2], tree, 3, 3)
    want = 0.9 * np.log(np.array([0.375, 0.125, 0.5]) + 1e-6)
    assert np.allclose(got[0], want, rtol=1e-6, atol=1e-6)


def test_tree_scores_of_one_leaf_is_tempered_softmax():
    rng = np.random.default_rng(1)
    s = rng.standard_normal((6, 5)).astype(np.float32) * 3
    got = oracle.tree_scores([s], [1, 6, 5, 0, 1, 2, 3, 4], 1, 5)
    z = np.exp((s - s.max(1, keepdims=True)) / 0.9)
    want = 0.9 * np.log(z / z.sum(1, keepdims=True) + 1e-6)
    assert np.abs(got - want).max() < 2e-6


def test_tree_scores_map_a_permuted_leaf():
    """A leaf's map sends its outputs to any classes: the scores follow the map."""
    rng = np.random.default_rng(2)
    s = rng.standard_normal((4, 3)).astype(np.float32)
    got = oracle.tree_scores([s], [1, 4, 3, 2, 0, 1], 1, 3)
    ident = oracle.tree_scores([s], [1, 4, 3, 0, 1, 2], 1, 3)
    assert np.array_equal(got[:, [2, 0, 1]], ident)


class _Shapes:
    """What raw_entries reads from the device weights: the in-context and the column stages' sizes."""
    shape = {"layers": 12, "d": 512}
    rows_shape = {"col_blocks": 3, "e": 128, "inds": 128}


@pytest.mark.parametrize("classes,kv", [(10, 1), (37, 2), (3, 0)])
def test_raw_entries_names_and_sizes(classes, kv):
    """fit::raw_entries (src/fit.rs:224-241): meta [7], the tree, col_kv [features][digits][blocks][2][e][inds], then
    per node its query scales [layers][d] and every layer's stored bytes, full chunks then the rest (chunk at least 8)."""
    rows, features, chunk = 1000, 7, 300
    y = np.arange(rows) % classes
    plan = tcu.Plan.new(10, y, classes)
    ent = tcu.raw_entries(_Shapes(), "m3/", rows, features, chunk, kv, plan)
    names = [n for n, _, _ in ent]
    assert names[:3] == ["m3/meta", "m3/tree", "m3/col_kv"]
    assert ent[0][1:] == ("int32", [7]) and ent[1][1:] == ("int32", [len(plan.tree(rows))])
    assert ent[2][2] == [features, len(plan.bases), 3, 2, 128, 128]
    at = 3
    for i, nd in enumerate(plan.nodes):
        nr = rows if nd.rows is None else len(nd.rows)
        assert ent[at] == (f"m3/n{i}_scale", "float32", [12, 512])
        want = (nr // chunk) * oracle.record(kv, 512, chunk) + (oracle.record(kv, 512, nr % chunk) if nr % chunk else 0)
        for l in range(12):
            assert ent[at + 1 + l] == (f"m3/n{i}_kv{l}", "uint8", [want])
        at += 13
    assert at == len(ent)
