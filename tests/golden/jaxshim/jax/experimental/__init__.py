from . import shard_map  # noqa: F401
