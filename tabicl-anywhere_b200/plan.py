"""How a table is fitted when it has more classes than the model tells apart: fit::Plan (src/fit.rs:151-221).

The classes are split into a tree of in-context problems: an inner node tells groups of classes apart, a leaf the
classes of one group; every node is fitted on the training rows of its classes, with its own targets. The column
stage sees the class label as mixed-radix digits (`bases`). `tree()` is the integer form stored as `m{i}/tree`
and read back by predict::Cache::open (src/predict.rs:138-161).
"""
import math

import numpy as np


class Node:
    """fit::Node (src/fit.rs:136-149): training rows (None: all of them), targets as this node sees them, outputs,
    leaf flag and map (a leaf: the class of each output; an inner node: the node index of each group)."""

    def __init__(self, rows, y, k, leaf, map_):
        self.rows, self.y, self.k, self.leaf, self.map = rows, y, k, leaf, map_

    def __repr__(self):
        n = "all" if self.rows is None else len(self.rows)
        return f"Node(rows={n}, k={self.k}, leaf={self.leaf}, map={self.map})"


class Plan:
    def __init__(self, bases, nodes):
        self.bases, self.nodes = bases, nodes

    @staticmethod
    def new(max_classes, y, classes):
        """fit.rs:159-184: one leaf over every row when the classes fit the model (or it is a regressor,
        max_classes 0); otherwise balanced label digits and the tree grown from all rows."""
        y = np.asarray(y, dtype=np.float32)
        mx = int(max_classes)
        if mx == 0 or classes <= mx:
            return Plan([max(classes, 1)], [Node(None, y, classes, True, list(range(classes)))])
        digits = int(math.ceil(math.log(classes) / math.log(mx)))
        k = min(int(math.ceil(classes ** (1.0 / digits))), mx)
        bases = [k] * digits
        product = k ** digits
        for i in range(len(bases)):
            if product >= classes:
                break
            if bases[i] < mx:
                product = product // bases[i] * (bases[i] + 1)
                bases[i] += 1
        nodes = []
        Plan._grow(mx, y, list(range(len(y))), nodes)
        return Plan(bases, nodes)

    @staticmethod
    def _grow(mx, y, rows, nodes):
        """fit.rs:186-215: a leaf when this node's classes fit, else an inner node over at most `mx` groups of
        consecutive classes (sizes as even as they go, larger first), each grown in turn."""
        labels = [int(y[r]) for r in rows]
        classes = sorted(set(labels))
        index = {c: i for i, c in enumerate(classes)}
        at = len(nodes)
        if len(classes) <= mx:
            ys = np.array([index[c] for c in labels], dtype=np.float32)
            nodes.append(Node(rows, ys, len(classes), True, classes))
            return at
        groups = min(-(-len(classes) // mx), mx)
        group_of = [0] * len(classes)
        pos, left = 0, len(classes)
        for g in range(groups):
            size = -(-left // (groups - g))
            group_of[pos:pos + size] = [g] * size
            pos += size
            left -= size
        ys = np.array([group_of[index[c]] for c in labels], dtype=np.float32)
        nodes.append(Node(list(rows), ys, groups, False, []))
        for g in range(groups):
            sub = [r for r, yg in zip(rows, ys) if int(yg) == g]
            child = Plan._grow(mx, y, sub, nodes)
            nodes[at].map.append(child)
        return at

    def tree(self, total_rows):
        """fit.rs:217-220: per node leaf, rows, k, map[0..k], as int32."""
        out = []
        for n in self.nodes:
            out += [int(n.leaf), total_rows if n.rows is None else len(n.rows), n.k] + [int(v) for v in n.map]
        return np.array(out, dtype=np.int32)
