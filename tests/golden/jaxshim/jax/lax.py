import numpy as _np


def square(x):
    return x * x


def rsqrt(x):
    return (_np.float32(1.0) / _np.sqrt(x)).astype(x.dtype)


def dot_general(x, w, dimension_numbers, preferred_element_type=None, precision=None):
    (cx, cw), (bx, bw) = dimension_numbers
    assert tuple(bx) == () and tuple(bw) == () and tuple(cw) == (0,) and tuple(cx) == (x.ndim - 1,)
    r = _np.matmul(_np.asarray(x, _np.float32), _np.asarray(w, _np.float32))
    return r.astype(preferred_element_type or _np.result_type(x.dtype, w.dtype))


def with_sharding_constraint(x, sharding):
    return x


def dynamic_update_slice(operand, update, start_indices):
    out = operand.copy()
    idx = []
    for d, s in enumerate(start_indices):
        s = int(_np.asarray(s))
        s = min(max(s, 0), operand.shape[d] - update.shape[d])
        idx.append(slice(s, s + update.shape[d]))
    out[tuple(idx)] = update
    return out


def top_k(x, k):
    x32 = _np.asarray(x, _np.float32)
    idx = _np.argsort(-x32, axis=-1, kind="stable")[..., :k].astype(_np.int32)
    return _np.take_along_axis(x, idx, axis=-1), idx


def axis_index(name):
    return 0


def psum(x, name):
    return x
