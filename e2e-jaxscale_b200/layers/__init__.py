"""Layer API of the reference (layers/*.py), backed by libjsx kernels."""
