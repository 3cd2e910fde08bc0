import numpy as _np


def PRNGKey(seed):
    return seed


class NoiseKey:
    """A key that carries the Gumbel noise of the next categorical draw (given by
    the caller, so a draw is reproducible outside JAX's generator)."""

    def __init__(self, gumbel):
        self.gumbel = gumbel


def split(key, num=2):
    return tuple(key for _ in range(num))


def categorical(key, logits, axis=-1):
    """jax.random.categorical's published form: argmax(logits + gumbel noise), the noise in
    the logits' dtype and the sum rounded to it; the first maximum wins."""
    z = logits + _np.asarray(key.gumbel).astype(logits.dtype)
    return _np.argmax(_np.asarray(z, _np.float32), axis=axis).astype(_np.int32)
