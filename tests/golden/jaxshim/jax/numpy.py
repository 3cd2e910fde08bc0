import ml_dtypes as _ml
import numpy as _np

bfloat16 = _ml.bfloat16
float32 = _np.float32
float16 = _np.float16
int32 = _np.int32
dtype = _np.dtype
ndarray = _np.ndarray


def asarray(x, dtype=None):
    return _np.asarray(x, dtype=dtype)


def array(x, dtype=None):
    return _np.array(x, dtype=dtype)


zeros = _np.zeros
ones = _np.ones
full = _np.full
arange = _np.arange
def where(cond, x=None, y=None):
    """jnp.where with JAX's weak typing: a Python scalar branch takes the other
    branch's dtype (numpy would promote a bf16 array and a float to float64)."""
    if x is None and y is None:
        return _np.where(cond)
    if isinstance(x, (int, float)) and isinstance(y, _np.ndarray):
        x = _np.asarray(x).astype(y.dtype)
    if isinstance(y, (int, float)) and isinstance(x, _np.ndarray):
        y = _np.asarray(y).astype(x.dtype)
    return _np.where(cond, x, y)


broadcast_to = _np.broadcast_to
expand_dims = _np.expand_dims
concatenate = _np.concatenate
split = _np.split
cos = _np.cos
sin = _np.sin
exp = _np.exp
take_along_axis = _np.take_along_axis
isin = _np.isin
cumsum = _np.cumsum


def argsort(a, axis=-1):
    return _np.argsort(a, axis=axis, kind="stable")  # jnp.argsort is stable
clip = _np.clip


def triu(m, k=0):
    m = _np.asarray(m)
    keep = _np.triu(_np.ones(m.shape, dtype=bool), k=k)
    return _np.where(keep, m, _np.zeros((), dtype=m.dtype)).astype(m.dtype)


def mean(x, axis=None, keepdims=False):
    return _np.mean(x, axis=axis, keepdims=keepdims, dtype=x.dtype)


def all(x):
    return _np.all(x)


def take(a, indices, axis=None):
    return _np.take(a, _np.asarray(indices), axis=axis)


def argmax(x, axis=None, keepdims=False):
    return _np.argmax(_np.asarray(x, _np.float32), axis=axis, keepdims=keepdims).astype(_np.int32)


def einsum(spec, *ops, preferred_element_type=None, precision=None):
    out_dtype = _np.result_type(*[o.dtype for o in ops])
    r = _np.einsum(spec, *[_np.asarray(o, _np.float32) for o in ops], dtype=_np.float32)
    return r.astype(preferred_element_type or out_dtype)


transpose = _np.transpose
swapaxes = _np.swapaxes


def matmul(a, b, preferred_element_type=None, precision=None):
    """jnp.matmul on bf16 operands: fp32-accumulated product, result in the operands' dtype."""
    out_dtype = _np.result_type(a.dtype, b.dtype)
    r = _np.matmul(_np.asarray(a, _np.float32), _np.asarray(b, _np.float32))
    return r.astype(preferred_element_type or out_dtype)
