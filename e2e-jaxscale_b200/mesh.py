"""Device mesh and tensor-parallel group (utils/mesh_utils.py:8-45).

The reference reshapes jax.devices() into a ("data", "tensor") or
("data", "expert", "tensor") mesh inside one controller process.  Here every
GPU is its own process (torchrun: RANK / WORLD_SIZE / LOCAL_RANK) and a
process's coordinates follow the same row-major reshape: rank r sits at
(r // tp, r % tp) in a 2-D mesh and at (r // (ep*tp), (r // tp) % ep, r % tp)
in a 3-D one.  The "tensor" axis is backed by a jsx_comm: a symmetric device
buffer per rank whose peers are mapped through CUDA IPC, used by the fused
row-parallel kernels.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from ._lib import JSX_ETIMEDOUT, JsxError, call


class Comm:
    """One rank's jsx_comm (include/jsx.h, jsx_comm_*).  tiles=True: the tile
    exchange of the wide row-parallel product (jsx_comm_create_tiles)."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int,
                 group=None, timeout_s: float = 5.0, tiles: bool = False):
        self.rank, self.world = rank, world
        self.max_tokens, self.hidden = max_tokens, hidden
        self.handle = ctypes.c_void_p()
        call("jsx_comm_create_tiles" if tiles else "jsx_comm_create", rank, world, max_tokens, hidden,
             int(timeout_s * 1e9), ctypes.byref(self.handle))
        if world > 1:
            buf = (ctypes.c_char * 64)()
            call("jsx_comm_ipc_handle", self.handle, buf)
            handles = [None] * world
            dist.all_gather_object(handles, bytes(buf), group=group)
            call("jsx_comm_open_peers", self.handle, b"".join(handles))
            dist.barrier(group=group)

    def check(self) -> None:
        """Raise JsxError(JSX_ETIMEDOUT) if any collective kernel gave up on a peer."""
        st = ctypes.c_int(0)
        call("jsx_comm_check", self.handle, ctypes.byref(st))
        if st.value != 0:
            raise JsxError(JSX_ETIMEDOUT, "jsx_comm_check", "a peer did not arrive in time")

    def close(self) -> None:
        if self.handle:
            call("jsx_comm_destroy", self.handle)
            self.handle = ctypes.c_void_p()


class Mesh:
    """Process-level view of the reference's named mesh."""

    def __init__(self, tp: int = 1, dp: int = 1, ep: int = 1, rank: int = 0, world: int = 1,
                 device=None):
        need = tp * dp * ep
        assert world >= need, (
            f"Need {need} devices (tp={tp}, dp={dp}, ep={ep}), but only {world} available.")
        self.tp, self.dp, self.ep = tp, dp, ep
        self.rank, self.world = rank, world
        if ep > 1:
            self.axis_names = ("data", "expert", "tensor")
            self.shape = {"data": dp, "expert": ep, "tensor": tp}
            self.coords = {"data": rank // (ep * tp), "expert": (rank // tp) % ep, "tensor": rank % tp}
        else:
            self.axis_names = ("data", "tensor")
            self.shape = {"data": dp, "tensor": tp}
            self.coords = {"data": rank // tp, "tensor": rank % tp}
        self.device = device
        self._groups = {}
        self._comms = {}

    @property
    def tp_rank(self) -> int:
        return self.coords["tensor"]

    def axis_ranks(self, axis: str, rank: int | None = None) -> list[int]:
        """Global ranks sharing every coordinate of `rank` except `axis`."""
        rank = self.rank if rank is None else rank
        names = self.axis_names
        sizes = [self.shape[n] for n in names]
        # coordinates of `rank` in row-major order
        c, rest = [], rank
        for s in reversed(sizes):
            c.append(rest % s)
            rest //= s
        c = list(reversed(c))
        i = names.index(axis)
        out = []
        for v in range(sizes[i]):
            cc = list(c)
            cc[i] = v
            r = 0
            for s, x in zip(sizes, cc):
                r = r * s + x
            out.append(r)
        return out

    def group(self, axis: str):
        """torch.distributed group of this rank along `axis` (every rank builds every group
        in the same order, as new_group requires)."""
        if axis in self._groups:
            return self._groups[axis]
        if not dist.is_initialized() or self.shape[axis] == 1:
            self._groups[axis] = None
            return None
        mine = None
        seen = set()
        for r in range(self.tp * self.dp * self.ep):
            ranks = tuple(self.axis_ranks(axis, r))
            if ranks in seen:
                continue
            seen.add(ranks)
            g = dist.new_group(list(ranks))
            if self.rank in ranks:
                mine = g
        self._groups[axis] = mine
        return mine

    def comm(self, max_tokens: int, hidden: int, timeout_s: float = 5.0) -> Comm | None:
        """The tensor-axis Comm (None when tp == 1)."""
        if self.tp == 1:
            return None
        key = (max_tokens, hidden)
        if key not in self._comms or not self._comms[key].handle:
            self._comms[key] = Comm(self.tp_rank, self.tp, max_tokens, hidden,
                                    group=self.group("tensor"), timeout_s=timeout_s)
        return self._comms[key]

    def comm_tiles(self, max_tokens: int, hidden: int, timeout_s: float = 5.0) -> Comm | None:
        """The tensor-axis tile-exchange Comm of the wide row-parallel product
        (prefill, many tokens); None when tp == 1."""
        if self.tp == 1:
            return None
        key = ("tiles", max_tokens, hidden)
        if key not in self._comms or not self._comms[key].handle:
            self._comms[key] = Comm(self.tp_rank, self.tp, max_tokens, hidden,
                                    group=self.group("tensor"), timeout_s=timeout_s, tiles=True)
        return self._comms[key]

    @property
    def moe_rank(self) -> int:
        """Index of this rank among the expert x tensor ranks of its data replica."""
        return self.coords.get("expert", 0) * self.tp + self.coords["tensor"]

    @property
    def moe_world(self) -> int:
        return self.ep * self.tp

    def comm_moe(self, max_tokens: int, hidden: int, timeout_s: float = 5.0) -> Comm | None:
        """Comm over the expert x tensor ranks of this data replica (None for one rank):
        the MoE layer's single exchange (psum over "expert" and the shared expert's
        tensor all-reduce, layers/moe.py:230 and :110-113)."""
        if self.moe_world == 1:
            return None
        key = ("moe", max_tokens, hidden)
        if key not in self._comms or not self._comms[key].handle:
            self._comms[key] = Comm(self.moe_rank, self.moe_world, max_tokens, hidden,
                                    group=self.group_moe(), timeout_s=timeout_s)
        return self._comms[key]

    def group_moe(self):
        """torch.distributed group of the expert x tensor ranks sharing this rank's data index."""
        if "moe" in self._groups:
            return self._groups["moe"]
        if not dist.is_initialized() or self.moe_world == 1:
            self._groups["moe"] = None
            return None
        mine = None
        span = self.ep * self.tp
        for d in range(self.dp):
            ranks = list(range(d * span, (d + 1) * span))
            g = dist.new_group(ranks)
            if self.rank in ranks:
                mine = g
        self._groups["moe"] = mine
        return mine

    def close(self) -> None:
        for c in self._comms.values():
            c.close()
        self._comms.clear()


def create_mesh(tp: int = 1, dp: int = 1, ep: int = 1) -> Mesh:
    """utils/mesh_utils.py:8-45.  Uses the torch.distributed world when initialised
    (one process per GPU), else a single process; binds this process to
    cuda:LOCAL_RANK when a GPU is present."""
    if dist.is_available() and dist.is_initialized():
        rank, world = dist.get_rank(), dist.get_world_size()
    else:
        rank, world = 0, 1
    device = None
    if torch.cuda.is_available():
        local = int(os.environ.get("LOCAL_RANK", rank % max(1, torch.cuda.device_count())))
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    return Mesh(tp=tp, dp=dp, ep=ep, rank=rank, world=world, device=device)
