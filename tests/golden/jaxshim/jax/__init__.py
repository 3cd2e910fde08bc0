"""numpy stand-in for the subset of jax used by the reference (see README.txt)."""
import numpy as _np

from . import experimental, lax, nn, numpy, random, sharding, tree_util  # noqa: F401

Array = _np.ndarray


def jit(fun=None, **kwargs):
    if fun is None:
        return lambda f: f
    return fun


def block_until_ready(x):
    return x


def devices():
    return ["cpu:0"]
