"""mlx.utils stand-in."""


def tree_flatten(tree, prefix="", is_leaf=None):
    out = []
    if isinstance(tree, dict):
        for k, v in tree.items():
            out += tree_flatten(v, f"{prefix}.{k}" if prefix else str(k), is_leaf)
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            out += tree_flatten(v, f"{prefix}.{i}" if prefix else str(i), is_leaf)
    else:
        out.append((prefix, tree))
    return out
