"""Data-parallel training of PackR layers: gradient reduce-scatter, 8-bit AdamW
on a 1/N shard of the optimizer state per rank, parameter all-gather.

The reference has no distributed code; this is the one parallel strategy the
B200 build adds (one process per GPU, NCCL over NVLink/NVSwitch).

Layout.  The trainable parameters (W_f, lut, bias_f, and any other tensors
passed in) are re-homed into flat buffers ("buckets"), one dtype per bucket,
filled in parameter order up to `bucket_bytes` (a larger parameter gets a
bucket of its own).  Each parameter starts at a multiple of 256 elements, so
the 256-element quantisation blocks of the 8-bit state never straddle two
parameters, and every bucket is padded to a multiple of 256 * world_size so
each rank's shard of it is a whole number of blocks.  A parameter's `.data`
becomes a view of its bucket, so the all-gather writes the updated values in
place.

Step (identical collective sequence on every rank), per bucket:
  1. the gradients land in the bucket's flat gradient buffer: each parameter
     carries `_packr_grad_sink = (flat_grad, offset)`, PackRLinear's backward
     writes dW_f straight into that slice while .grad is None, other
     gradients are copied (zeros where None)
  2. reduce_scatter_tensor(op=AVG)   -> this rank's averaged gradient shard
  3. packr_adam8_multi over the parameter sub-ranges of the shard (the same
     per-block arithmetic as CUDA8BitAdam, so the result equals the
     single-process step on the averaged gradient)
  4. every rank receives the new parameters:
     transport "push" (one node, NCCL, CUDA; "auto" takes it for 2-4
       ranks): a rank's buckets sit in one cudaMalloc arena that the other
       ranks map by CUDA IPC; packr_adam8_multi_push
       stores each updated value into the rank's own bucket and into every
       other rank's copy over NVLink, and one one-element all-reduce after
       the last bucket orders those stores before any rank's next read.  No
       all-gather kernel runs, so nothing competes for SMs with the next
       step's persistent GEMMs or with AdamW itself;
     transport "nccl": all_gather_into_tensor per bucket.
With overlap_grad_reduce=True (world_size > 1) step 2 of a bucket is issued
asynchronously from a post-accumulate-grad hook as soon as the last gradient
of the bucket is produced, so it runs on NCCL's stream while the backward of
earlier layers continues; step() then waits for it.  That assumes one
backward per step: wrap the earlier micro-batches of gradient accumulation in
`with opt.no_sync():`.  With world_size 1 the collectives are skipped and the
optimizer reads the flat gradient buffer itself.
"""
from __future__ import annotations

import contextlib
import ctypes
import socket
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

BLOCK = 256
AUTO_PUSH_MAX_RANKS = 4


@dataclass
class _Slot:
    param: torch.Tensor
    offset: int   # element offset in the bucket (multiple of BLOCK)
    numel: int


@dataclass
class _Bucket:
    dtype: torch.dtype
    slots: list = field(default_factory=list)
    total: int = 0
    flat: torch.Tensor | None = None
    grad: torch.Tensor | None = None
    shard_grad: torch.Tensor | None = None
    m: torch.Tensor | None = None
    v: torch.Tensor | None = None
    ms: torch.Tensor | None = None
    vs: torch.Tensor | None = None
    entries: list = field(default_factory=list)  # (p_view, g_view, m, v, ms, vs)
    peer_ptrs: list = field(default_factory=list)  # push: per entry, its address in every other rank's bucket
    arena_off: int = 0                            # push: byte offset of `flat` in the rank's arena
    ready: int = 0                                # gradients produced since the last step (overlap mode)
    work: object = None                           # pending reduce-scatter


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class _DeviceBuffer:
    """A cudaMalloc allocation (packr_device_alloc: exportable by CUDA IPC as
    a whole) with the CUDA array interface, so torch.as_tensor views it; the
    tensor keeps this object, and so the allocation, alive."""

    def __init__(self, nbytes: int, device: torch.device):
        from . import _lib
        self._lib = _lib.load()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check("packr_device_alloc", self._lib.packr_device_alloc(nbytes, ctypes.byref(ptr)))
        self.ptr, self.nbytes, self.device = ptr.value, nbytes, device
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (self.ptr, False),
                                         "version": 3, "strides": None}

    def tensor(self, dtype: torch.dtype, numel: int, offset: int = 0) -> torch.Tensor:
        """Zeroed [numel] `dtype` view starting `offset` bytes in."""
        esz = torch.empty((), dtype=dtype).element_size()
        t = torch.as_tensor(self, device=self.device)[offset:offset + numel * esz]
        return t.view(dtype).zero_()

    def handle(self) -> bytes:
        from . import _lib
        h = ctypes.create_string_buffer(_lib.PACKR_IPC_HANDLE_BYTES)
        _lib.check("packr_ipc_export", self._lib.packr_ipc_export(ctypes.c_void_p(self.ptr), h))
        return h.raw

    def __del__(self):
        if getattr(self, "ptr", None):
            try:
                with torch.cuda.device(self.device):
                    self._lib.packr_device_free(ctypes.c_void_p(self.ptr))
            except Exception:  # interpreter shutdown: the CUDA context may already be gone
                pass
            self.ptr = None


class ShardedAdam8:
    """ZeRO-1 data-parallel 8-bit AdamW over `params` (same device).

    adam_fn(entries, lr, b1, b2, eps, bc1, bc2, wd) performs the 8-bit AdamW
    update on a list of (p, g, m, v, m_scale, v_scale) tensors; the default is
    the sm_100a kernel (packr_b200.cuda_adam.adam8_launch).
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, process_group=None,
                 adam_fn=None, bucket_bytes: int = 32 << 20, overlap_grad_reduce: bool = False,
                 transport: str = "auto"):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("ShardedAdam8: no trainable parameters")
        self.betas, self.eps, self.weight_decay = betas, eps, weight_decay
        # one group, so that LR controllers (VelvetController, schedulers) can
        # set group["lr"] as they do on a torch optimizer
        self.param_groups = [{"params": self.params, "lr": lr}]
        self.state: dict = {}  # the 8-bit state lives in the buckets (state_dict, v_means)
        self.pg = process_group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(self.pg)
            self.rank = dist.get_rank(self.pg)
        else:
            self.world, self.rank = 1, 0
        if transport not in ("auto", "push", "nccl"):
            raise ValueError(f"ShardedAdam8: transport must be 'auto', 'push' or 'nccl', not {transport!r}")
        custom_adam = adam_fn is not None
        if adam_fn is None:
            from .cuda_adam import adam8_launch
            adam_fn = adam8_launch
        self.adam_fn = adam_fn
        self.device = self.params[0].device
        self.transport = "nccl"
        # "auto" takes the push transport up to AUTO_PUSH_MAX_RANKS ranks, the
        # sizes it was measured at; above that every GPU must take in 7/8 of
        # the parameters either way (pushes or all-gather), and the all-gather
        # is the measured path there
        if self.world > 1 and (transport == "push" or (transport == "auto" and self.world <= AUTO_PUSH_MAX_RANKS)):
            why = self._push_unavailable(custom_adam)
            if why is None:
                self.transport = "push"
            elif transport == "push":
                raise RuntimeError(f"ShardedAdam8: transport 'push' unavailable: {why}")
        self.step_count = 0
        self.buckets: list[_Bucket] = []
        open_bucket: dict[torch.dtype, _Bucket] = {}
        for p in self.params:
            if p.device != self.device:
                raise ValueError("ShardedAdam8: all parameters must be on one device")
            b = open_bucket.get(p.dtype)
            if b is None or (b.slots and (b.total + p.numel()) * p.element_size() > bucket_bytes):
                b = _Bucket(p.dtype)
                self.buckets.append(b)
                open_bucket[p.dtype] = b
            b.slots.append(_Slot(p, b.total, p.numel()))
            b.total = _round_up(b.total + p.numel(), BLOCK)
        self._index = {id(p): i for i, p in enumerate(self.params)}
        self._bucket_of = {}
        for b in self.buckets:
            b.total = _round_up(max(b.total, 1), BLOCK * self.world)
        # push: every bucket of this rank in one cudaMalloc arena, so that one
        # IPC handle per rank maps all of them
        self._arena = None
        if self.transport == "push":
            off = 0
            for b in self.buckets:
                b.arena_off = off
                off = _round_up(off + b.total * torch.empty((), dtype=b.dtype).element_size(), 256)
            self._arena = _DeviceBuffer(off, self.device)
        for b in self.buckets:
            self._build(b)
            for s in b.slots:
                self._bucket_of[id(s.param)] = b
        self._peer_maps: list[int] = []
        if self.transport == "push" and not self._connect_peers():
            self.transport = "nccl"
        self._barrier = torch.zeros(1, dtype=torch.int32, device=self.device) if self.transport == "push" else None
        self.overlap = bool(overlap_grad_reduce) and self.world > 1
        self._sync = True
        if self.overlap:
            for p in self.params:
                p.register_post_accumulate_grad_hook(self._on_grad)

    # -------------------------------------------------------------- transport
    def _push_unavailable(self, custom_adam: bool):
        """None when every rank can take the push transport, else the reason
        (the same answer on every rank: one all_gather_object)."""
        local = None
        if custom_adam:
            local = "a custom adam_fn"
        elif dist.get_backend(self.pg) != "nccl" or self.device.type != "cuda":
            local = "needs the NCCL backend and CUDA parameters"
        elif self.world - 1 > 7:
            local = "more than 8 ranks"
        info = [None] * self.world
        dist.all_gather_object(info, (socket.gethostname(), local), group=self.pg)
        reasons = [r for _, r in info if r is not None]
        if reasons:
            return reasons[0]
        if len({h for h, _ in info}) != 1:
            return "ranks on more than one node"
        return None

    def _connect_peers(self) -> bool:
        """Exchanges the arenas' IPC handles and maps every other rank's
        arena; True when every rank mapped all of them (an all-reduce of the
        outcome, so the ranks agree)."""
        from . import _lib
        lib = _lib.load()
        try:
            mine = (self._arena.handle(), [b.arena_off for b in self.buckets])
        except RuntimeError:
            mine = None
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.pg)
        if any(e is None or e[1] != mine[1] for e in everyone):
            return False  # the same answer on every rank; nothing mapped yet
        bases = {}  # rank -> mapped address of its arena
        ok = True
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    continue
                h = everyone[q][0]
                ptr = ctypes.c_void_p()
                if lib.packr_ipc_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(ptr)) != 0:
                    ok = False
                    break
                self._peer_maps.append(ptr.value)
                bases[q] = ptr.value
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.pg)
        if int(flag.item()) == 0:
            self.close()
            return False
        for b in self.buckets:
            esz = b.flat.element_size()
            b.peer_ptrs = [[bases[q] + b.arena_off + off * esz for q in range(self.world) if q != self.rank]
                           for off in b._entry_offsets]
        return True

    def close(self) -> None:
        """Unmaps the other ranks' buckets (push transport); the optimizer
        then uses the all-gather.  Collective with the push transport: every
        rank calls it, and it returns when every rank has unmapped, so that no
        rank frees a bucket another rank still maps."""
        from . import _lib
        was_push = self.transport == "push" or bool(self._peer_maps)
        if self._peer_maps:
            lib = _lib.load()
            torch.cuda.synchronize(self.device)
            with torch.cuda.device(self.device):
                for ptr in self._peer_maps:
                    lib.packr_ipc_close(ctypes.c_void_p(ptr))
            self._peer_maps = []
        for b in self.buckets:
            b.peer_ptrs = []
        self.transport = "nccl"
        self._barrier = None
        if was_push and self.world > 1:
            dist.barrier(group=self.pg)

    # -------------------------------------------------------------- layout
    def _build(self, b: _Bucket) -> None:
        total = b.total
        if self._arena is not None:
            b.flat = self._arena.tensor(b.dtype, total, b.arena_off)
        else:
            b.flat = torch.zeros(total, dtype=b.dtype, device=self.device)
        b.grad = torch.zeros(total, dtype=b.dtype, device=self.device)
        for s in b.slots:
            b.flat[s.offset:s.offset + s.numel].copy_(s.param.detach().reshape(-1))
            s.param.data = b.flat[s.offset:s.offset + s.numel].view_as(s.param)
            s.param._packr_grad_sink = (b.grad, s.offset)
        shard = total // self.world
        s0 = self.rank * shard
        b.shard_grad = b.grad if self.world == 1 else torch.zeros(shard, dtype=b.dtype, device=self.device)
        b.m = torch.zeros(shard, dtype=torch.int8, device=self.device)
        b.v = torch.zeros(shard, dtype=torch.int8, device=self.device)
        b.ms = torch.ones(shard // BLOCK, dtype=torch.float32, device=self.device)
        b.vs = torch.ones(shard // BLOCK, dtype=torch.float32, device=self.device)
        # parameter sub-ranges inside this rank's shard; both ends of each
        # range are 256-aligned except a parameter's own last element
        b._entry_offsets = []
        for s in b.slots:
            a, e = max(s.offset, s0), min(s.offset + s.numel, s0 + shard)
            if a >= e:
                continue
            la, le = a - s0, e - s0
            ba, be = la // BLOCK, (le + BLOCK - 1) // BLOCK
            b.entries.append((b.flat[a:e], b.shard_grad[la:le], b.m[la:le], b.v[la:le], b.ms[ba:be], b.vs[ba:be]))
            b._entry_offsets.append(a)

    @property
    def lr(self) -> float:
        return self.param_groups[0]["lr"]

    @lr.setter
    def lr(self, value: float) -> None:
        self.param_groups[0]["lr"] = value

    @property
    def shard_numel(self) -> int:
        return sum(b.total // self.world for b in self.buckets)

    def bucket_of(self, param: torch.Tensor) -> _Bucket:
        return self._bucket_of[id(param)]

    # -------------------------------------------------------------- gradients
    def _gather_grads(self, b: _Bucket) -> None:
        for s in b.slots:
            dst = b.grad[s.offset:s.offset + s.numel]
            if s.param.grad is None:
                dst.zero_()
            elif s.param.grad.data_ptr() != dst.data_ptr():  # not already the slice
                dst.copy_(s.param.grad.reshape(-1))

    def _launch_reduce(self, b: _Bucket) -> None:
        self._gather_grads(b)
        if self.world > 1:
            b.work = dist.reduce_scatter_tensor(b.shard_grad, b.grad, op=dist.ReduceOp.AVG, group=self.pg,
                                                async_op=True)
        else:
            b.work = True

    def _on_grad(self, param: torch.Tensor) -> None:
        if not self._sync:
            return
        b = self._bucket_of[id(param)]
        b.ready += 1
        if b.ready == len(b.slots) and b.work is None:
            self._launch_reduce(b)

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside do not start the gradient reduce-scatter
        (the earlier micro-batches of gradient accumulation)."""
        prev, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = prev

    # -------------------------------------------------------------- step
    @torch.no_grad()
    def step(self) -> None:
        self.step_count += 1
        b1, b2 = self.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        for b in self.buckets:  # the same collective order on every rank
            if b.work is None:
                self._launch_reduce(b)
        gathers = []
        push = self.transport == "push"
        if push:
            from .cuda_adam import adam8_launch_push
        for b in self.buckets:
            if self.world > 1:
                b.work.wait()
            b.work = None
            b.ready = 0
            if push:
                if b.entries:
                    adam8_launch_push(b.entries, b.peer_ptrs, self.lr, b1, b2, self.eps, bc1, bc2,
                                      self.weight_decay)
                continue
            if b.entries:
                self.adam_fn(b.entries, self.lr, b1, b2, self.eps, bc1, bc2, self.weight_decay)
            if self.world > 1:
                shard = b.total // self.world
                mine = b.flat[self.rank * shard:(self.rank + 1) * shard]
                src = mine if self.device.type == "cuda" else mine.clone()
                gathers.append(dist.all_gather_into_tensor(b.flat, src, group=self.pg, async_op=True))
        if push:
            # every rank's stores into the others' buckets precede (stream
            # order, system-scope fence at the end of each AdamW kernel) its
            # part of this all-reduce, which every rank's stream waits for
            dist.all_reduce(self._barrier, group=self.pg)
        for w in gathers:
            w.wait()

    @torch.no_grad()
    def v_means(self) -> dict:
        """{id(param): mean of the dequantised second moment} over the whole
        parameter, for VelvetController.  Each rank sums the codes x block
        scale of the parameter slices in its shard (one packr_state_v_sums
        launch), one all-reduce of the per-parameter sums (the same call on
        every rank) combines the shards, one copy brings them to the host."""
        from .velvet import state_v_sums
        slices, where = [], []
        for i, p in enumerate(self.params):
            b = self._bucket_of[id(p)]
            shard = b.total // self.world
            s0 = self.rank * shard
            slot = next(s for s in b.slots if s.param is p)
            a, e = max(slot.offset, s0), min(slot.offset + slot.numel, s0 + shard)
            if a < e:
                slices.append((b.v, b.vs, a - s0, e - a, BLOCK))
                where.append(i)
        sums = torch.zeros(len(self.params), dtype=torch.float64, device=self.device)
        if slices:
            sums.index_copy_(0, torch.tensor(where, device=self.device), state_v_sums(slices, self.device))
        if self.world > 1:
            dist.all_reduce(sums, group=self.pg)
        n = torch.tensor([max(p.numel(), 1) for p in self.params], dtype=torch.float64, device=self.device)
        return dict(zip((id(p) for p in self.params), (sums / n).cpu().tolist()))

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def state_dict(self) -> dict:
        """This rank's shard of the 8-bit state (int8 m/v, f32 block scales), per bucket."""
        return {"step": self.step_count, "world": self.world, "rank": self.rank,
                "buckets": [{"dtype": str(b.dtype), "m": b.m, "v": b.v, "m_scale": b.ms, "v_scale": b.vs}
                            for b in self.buckets]}

    # ----------------------------------------------------- consolidated state
    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        """All ranks' shards of a bucket buffer, concatenated in rank order."""
        if self.world == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous(), group=self.pg)
        return torch.cat(parts)

    @torch.no_grad()
    def consolidated_state_dict(self) -> dict:
        """The whole optimizer state in CUDA8BitAdam.state_dict()'s format
        (per parameter, keyed by its position in the parameter list; m/v int8
        [numel], m_scale/v_scale f32 [ceil(numel / 256)]), independent of the
        world size: it loads into CUDA8BitAdam or into a ShardedAdam8 over any
        number of ranks.  Collective: every rank calls it and gets the whole
        dict.  A parameter's blocks are its own blocks in the flat buffer
        (parameters start at multiples of 256), so nothing is re-quantised."""
        state = {}
        for b in self.buckets:
            m, v, ms, vs = (self._gather(t) for t in (b.m, b.v, b.ms, b.vs))
            for s in b.slots:
                i = self._index[id(s.param)]
                b0, nb = s.offset // BLOCK, (s.numel + BLOCK - 1) // BLOCK
                state[i] = {"m": m[s.offset:s.offset + s.numel].clone(), "v": v[s.offset:s.offset + s.numel].clone(),
                            "m_scale": ms[b0:b0 + nb].clone(), "v_scale": vs[b0:b0 + nb].clone()}
        group = {"lr": self.lr, "betas": tuple(self.betas), "eps": self.eps, "weight_decay": self.weight_decay,
                 "params": list(range(len(self.params)))}
        return {"state": state, "param_groups": [group], "packr_step_count": self.step_count}

    @torch.no_grad()
    def load_consolidated_state_dict(self, sd: dict) -> None:
        """Loads a consolidated_state_dict() (or CUDA8BitAdam.state_dict()
        over the same parameters in the same order): each rank copies the
        ranges of its own shard."""
        state = sd["state"]
        if len([i for g in sd["param_groups"] for i in g["params"]]) != len(self.params):
            raise ValueError("ShardedAdam8.load_consolidated_state_dict: different number of parameters")
        for b in self.buckets:
            shard = b.total // self.world
            s0 = self.rank * shard
            for s in b.slots:
                st = state.get(self._index[id(s.param)])
                a, e = max(s.offset, s0), min(s.offset + s.numel, s0 + shard)
                if a >= e:
                    continue
                la, le = a - s0, e - s0
                ba, be = la // BLOCK, (le + BLOCK - 1) // BLOCK
                pa, pb = (a - s.offset) // BLOCK, (e - s.offset + BLOCK - 1) // BLOCK
                if st is None:  # never stepped: the initial state
                    b.m[la:le] = 0
                    b.v[la:le] = 0
                    b.ms[ba:be] = 1.0
                    b.vs[ba:be] = 1.0
                    continue
                if st["m"].numel() != s.numel or st["m_scale"].numel() != (s.numel + BLOCK - 1) // BLOCK:
                    raise ValueError("ShardedAdam8.load_consolidated_state_dict: state shape mismatch")
                b.m[la:le].copy_(st["m"][a - s.offset:e - s.offset])
                b.v[la:le].copy_(st["v"][a - s.offset:e - s.offset])
                b.ms[ba:be].copy_(st["m_scale"][pa:pb])
                b.vs[ba:be].copy_(st["v_scale"][pa:pb])
        self.step_count = int(sd.get("packr_step_count", self.step_count))
        self.lr = sd["param_groups"][0]["lr"]

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["rank"] != self.rank:
            raise ValueError("ShardedAdam8.load_state_dict: saved for a different world size / rank")
        if len(sd["buckets"]) != len(self.buckets):
            raise ValueError("ShardedAdam8.load_state_dict: saved with a different bucket layout")
        self.step_count = int(sd["step"])
        for b, s in zip(self.buckets, sd["buckets"]):
            if s["dtype"] != str(b.dtype) or s["m"].numel() != b.m.numel():
                raise ValueError("ShardedAdam8.load_state_dict: saved with a different bucket layout")
            b.m.copy_(s["m"]); b.v.copy_(s["v"]); b.ms.copy_(s["m_scale"]); b.vs.copy_(s["v_scale"])
