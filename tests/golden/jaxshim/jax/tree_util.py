def register_pytree_node(cls, flatten, unflatten):
    return None


def tree_flatten(x):
    return [x], None


def tree_unflatten(d, leaves):
    return leaves[0]
