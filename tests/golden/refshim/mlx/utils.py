"""CPU stand-in for ``mlx.utils`` tree helpers (test infrastructure only).

``tree_flatten`` turns nested dicts/lists into ``("a.b.0.c", leaf)`` pairs;
``tree_unflatten`` inverts it, making lists where every key of a level is an
integer, as MLX documents.
"""

from __future__ import annotations


def tree_flatten(tree, prefix: str = "", is_leaf=None):
    out = []
    if is_leaf is not None and is_leaf(tree):
        return [(prefix[1:] if prefix.startswith(".") else prefix, tree)]
    if isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            out.extend(tree_flatten(v, f"{prefix}.{i}", is_leaf))
        return out
    if isinstance(tree, dict):
        for k, v in tree.items():
            out.extend(tree_flatten(v, f"{prefix}.{k}", is_leaf))
        return out
    return [(prefix[1:] if prefix.startswith(".") else prefix, tree)]


def tree_unflatten(tree):
    if len(tree) == 1 and tree[0][0] == "":
        return tree[0][1]
    try:
        int(tree[0][0].split(".", maxsplit=1)[0])
        is_list = True
    except ValueError:
        is_list = False
    children = {}
    for key, value in tree:
        current, *rest = key.split(".", maxsplit=1)
        children.setdefault(current, []).append((rest[0] if rest else "", value))
    if is_list:
        out = []
        for i, k in sorted((int(k), k) for k in children):
            while len(out) < i:
                out.append({})
            out.append(tree_unflatten(children[k]))
        return out
    return {k: tree_unflatten(v) for k, v in children.items()}


def tree_map(fn, tree, *rest, is_leaf=None):
    if is_leaf is not None and is_leaf(tree):
        return fn(tree, *rest)
    if isinstance(tree, (list, tuple)):
        return type(tree)(tree_map(fn, c, *[r[i] for r in rest], is_leaf=is_leaf) for i, c in enumerate(tree))
    if isinstance(tree, dict):
        return {k: tree_map(fn, c, *[r[k] for r in rest], is_leaf=is_leaf) for k, c in tree.items()}
    return fn(tree, *rest)
