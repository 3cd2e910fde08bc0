import numpy as _np


def sigmoid(x):
    x32 = _np.asarray(x, _np.float32)
    return (_np.float32(1.0) / (_np.float32(1.0) + _np.exp(-x32))).astype(x.dtype)


def silu(x):
    return x * sigmoid(x)


def softmax(x, axis=-1):
    x32 = _np.asarray(x, _np.float32)
    e = _np.exp(x32 - x32.max(axis=axis, keepdims=True))
    return (e / e.sum(axis=axis, keepdims=True, dtype=_np.float32)).astype(x.dtype)


def dot_product_attention(query, key, value, bias=None, mask=None, *, scale=None, is_causal=False,
                          implementation=None, **kw):
    B, T, N, H = query.shape
    K = key.shape[2]
    g = N // K
    q = _np.asarray(query, _np.float32).reshape(B, T, K, g, H)
    k = _np.asarray(key, _np.float32)
    logits = _np.einsum("btkgh,bskh->bkgts", q, k, dtype=_np.float32)
    logits = logits * _np.float32(scale if scale is not None else H ** -0.5)
    if bias is not None:
        b = _np.asarray(bias, _np.float32)  # [B or 1, N or 1, T, S]
        b = b.reshape(b.shape[0], 1 if b.shape[1] == 1 else K, 1 if b.shape[1] == 1 else g, *b.shape[2:])
        logits = logits + b
    probs = softmax(logits, axis=-1).astype(key.dtype)
    out = _np.einsum("bkgts,bskh->btkgh", _np.asarray(probs, _np.float32), _np.asarray(value, _np.float32),
                     dtype=_np.float32)
    return out.reshape(B, T, N, H).astype(query.dtype)
