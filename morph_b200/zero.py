"""ZeRO-1 sharded AdamW across the GPUs of one node (one process per GPU).

The reference is single-process; this is the one parallel strategy the B200
build adds. The flat parameter space (all tensors in order) is cut into
16-element-aligned chunks dealt round-robin: in round k, rank r owns chunk
k*N + r. Rank r keeps the FP32 master weights and the two moments of its
chunks; every rank holds the full low-precision (BF16) weights the model
computes with. One step:

  1. kernel 2 over this rank's slice of the (already reduced) gradients
     writes the 16-byte record {sum of squares, nonfinite} (FP64);
  2. all_reduce(SUM) of that record, so every rank takes the same skip /
     clip decision;
  3. the one-CTA finalize (clip coefficient, clocks, step scalars);
  4. per round k: kernel 1 updates this rank's chunk of round k and writes its
     BF16 copy into place; then all_gather_into_tensor of round k's N chunks
     (one contiguous block of the flat buffer, in place) starts on NCCL's
     stream while round k + 1 is updated.

Only those two collectives exist (NCCL over NVLink on B200 nodes). The kernel
calls go through a backend object: ``CudaZeroBackend`` (the C-ABI library) is
the only one this package provides.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib
from .optim import StepEngine, TILE

ALIGN = 16


def chunk_size(total: int, world: int, rounds: int, align: int = ALIGN) -> int:
    """Chunk length (elements) so that rounds x world chunks cover total."""
    cs = -(-total // (world * rounds))
    return -(-cs // align) * align


def rank_chunks(total: int, world: int, rank: int, rounds: int, cs: int):
    """(round, lo, hi) of the flat ranges this rank owns (possibly empty)."""
    out = []
    for k in range(rounds):
        lo = min(total, (k * world + rank) * cs)
        hi = min(total, lo + cs)
        out.append((k, lo, hi))
    return out


def shard_pieces(sizes, lo, hi):
    """(tensor index, offset in tensor, offset from lo, length) of every piece of
    the tensors inside [lo, hi) of the flat space."""
    pieces, off = [], 0
    for i, n in enumerate(sizes):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            pieces.append((i, a - off, a - lo, b - a))
        off += n
    return pieces


class _CudaArray:
    """__cuda_array_interface__ over a raw device pointer (no ownership)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class PeerBuffer:
    """A device buffer of this rank that every rank of the group (one node) has
    mapped: ``tensor`` is the local view, ``deltas`` the byte offsets from a
    local address to the same element in each other rank's buffer."""

    def __init__(self, nbytes, device, group=None):
        self.device = torch.device(device)
        self.group = group
        lib = _lib.lib()
        handle = (ctypes.c_uint8 * 64)()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.mb_ipc_alloc(int(nbytes), ctypes.byref(ptr), handle), "mb_ipc_alloc")
        self.ptr = ptr.value
        self.nbytes = int(nbytes)
        handles = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, bytes(handle), group=group)
        me = dist.get_rank(group)
        world = len(handles)
        self.peers = []
        try:
            with torch.cuda.device(self.device):
                # peers in the order me+1, me+2, ...: a kernel storing to its peers
                # in list order then starts on a different GPU on every rank, so no
                # GPU's links receive everyone's first stores at once
                for k in range(1, world):
                    h = handles[(me + k) % world]
                    pp = ctypes.c_void_p()
                    _lib.check(lib.mb_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(pp)),
                               "mb_ipc_open")
                    self.peers.append(pp.value)
        except Exception:
            with torch.cuda.device(self.device):
                for pp in self.peers:
                    lib.mb_ipc_close(ctypes.c_void_p(pp))
                lib.mb_ipc_free(ctypes.c_void_p(self.ptr))
            raise
        self.deltas = [pp - self.ptr for pp in self.peers]
        raw = torch.as_tensor(_CudaArray(self.ptr, self.nbytes // 2, "<i2"), device=self.device)
        self.tensor = raw.view(torch.bfloat16)

    def close(self):
        """Unmap the peers' buffers, wait for every rank, free this rank's."""
        if self.ptr is None:
            return
        lib = _lib.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for pp in self.peers:
                lib.mb_ipc_close(ctypes.c_void_p(pp))
        self.peers = []
        dist.barrier(group=self.group)  # no rank still maps this buffer
        self.tensor = None
        with torch.cuda.device(self.device):
            lib.mb_ipc_free(ctypes.c_void_p(self.ptr))
        self.ptr = None


class CudaZeroBackend:
    """Kernel calls of one ZeRO step on the rank's GPU (C-ABI library)."""

    def __init__(self, device, reserve_sms=0):
        self.device = torch.device(device)
        self.engine = StepEngine(self.device)
        self._plan = None
        self._round_tiles = []
        # CTAs of kernel 1 when some SMs are left to the concurrent all-gather
        # (kernel 1 runs 3 CTAs per SM at full occupancy)
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.max_ctas = 3 * max(1, sms - reserve_sms) if reserve_sms > 0 else 0

    def record(self) -> torch.Tensor:
        """The device record {sumsq, nonfinite} as a 2-element FP64 view."""
        return self.engine.state_buf[:16].view(torch.float64)

    def prepare(self, keys, entries, rounds, lr, betas, eps, weight_decay, grad_dtype, out_dtype):
        """entries are ordered by round; rounds[i] is entry i's round."""
        for k in keys:
            self.engine.slot(k, 0)
        groups = [(float(lr), float(betas[0]), float(betas[1]), float(eps), float(weight_decay), "torch")]
        self._plan = self.engine.prepare(entries, groups, _lib.dtype_code(grad_dtype), _lib.dtype_code(out_dtype),
                                         keys=keys)
        nr = (max(rounds) + 1) if rounds else 0
        tiles = [0] * (nr + 1)
        for e, r in zip(entries, rounds):
            tiles[r + 1] += (e[3].numel() + TILE - 1) // TILE
        for r in range(nr):
            tiles[r + 1] += tiles[r]
        self._round_tiles = tiles

    def finalize_opts(self, fin_flags, max_norm):
        self._fin = self.engine.finalize_opts(fin_flags, max_norm)

    def stats(self, fin_flags, max_norm):
        self.finalize_opts(fin_flags, max_norm)
        with torch.cuda.device(self.device):
            _lib.check(self.engine.lib.mb_grad_stats(ctypes.byref(self._plan), None, _lib.stream_handle()),
                       "mb_grad_stats")

    def finalize(self):
        with torch.cuda.device(self.device):
            _lib.check(self.engine.lib.mb_step_finalize(ctypes.byref(self._plan), ctypes.byref(self._fin),
                                                        _lib.stream_handle()), "mb_step_finalize")
        self.engine.max_clock += 1

    def apply_round(self, k, peer_deltas=None):
        """Kernel 1 on round k's tiles; with ``peer_deltas`` every low-precision
        value is also stored into the other ranks' buffers (fused all-gather)."""
        lo, hi = self._round_tiles[k], self._round_tiles[k + 1]
        with torch.cuda.device(self.device):
            if peer_deltas:
                arr = (ctypes.c_int64 * len(peer_deltas))(*peer_deltas)
                _lib.check(self.engine.lib.mb_adamw_apply_tiles_peers(
                    ctypes.byref(self._plan), lo, hi, 0, arr, len(peer_deltas), _lib.stream_handle()),
                    "mb_adamw_apply_tiles_peers")
            else:
                _lib.check(self.engine.lib.mb_adamw_apply_tiles(ctypes.byref(self._plan), lo, hi, self.max_ctas,
                                                                _lib.stream_handle()), "mb_adamw_apply_tiles")

    def last_step(self) -> dict:
        st = self.engine.read_state()
        return dict(norm=float(st.norm), skipped=bool(st.skip), status=int(st.status),
                    clip_coef=float(st.clip_coef))

    def skip_flag(self) -> int:
        """Device address of the step state's skip flag (kernels read it)."""
        return self.engine.state_buf.data_ptr() + _lib.StepState.skip.offset


class ZeroAdamW:
    """ZeRO-1 AdamW (torch AdamW arithmetic, decoupled weight decay).

    params: the model's FP32 tensors with identical initial values on every
    rank (only this rank's chunks are copied into the masters). After each
    ``step(grads)`` the full updated weights are in ``weights`` (one
    low-precision tensor per parameter, views of one flat buffer). ``rounds``
    is the number of update/all-gather rounds that overlap (1 on one GPU);
    ``reserve_sms`` SMs are left free of kernel 1 for NCCL's all-gather.

    ``sync`` (default: ``gate``) makes ``step`` wait for the step's device
    record and raise FloatingPointError at once when the gate refused it.
    With ``sync=False`` the step only enqueues work, so the host prepares the
    next step while this one runs; a refused step still changes nothing on
    any rank, and ``check()`` (or ``last_step()``) reports it later."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, *, max_norm=None,
                 clip_mode="torch", gate=False, low_precision=torch.bfloat16, process_group=None, device=None,
                 backend=None, rounds=8, reserve_sms=24, peer_writes="auto", sync=None):
        params = list(params)
        if not params:
            raise ValueError("ZeroAdamW needs parameters")
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else params[0].device
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.max_norm, self.clip_mode, self.gate = max_norm, clip_mode, gate
        self.sync = gate if sync is None else bool(sync)
        if clip_mode not in ("torch", "disk"):
            raise ValueError("clip_mode must be 'torch' or 'disk'")
        self.low_precision = low_precision
        self.shapes = [tuple(p.shape) for p in params]
        self.sizes = [p.numel() for p in params]
        self.total = sum(self.sizes)
        self.peer_writes = self._want_peers(peer_writes, backend)
        # peer writes replace the per-round all-gathers: one update launch stores everywhere
        self.rounds = 1 if self.world == 1 or self.peer_writes else max(1, int(rounds))
        self.cs = chunk_size(self.total, self.world, self.rounds)
        self.chunks = rank_chunks(self.total, self.world, self.rank, self.rounds, self.cs)
        # pieces: (tensor index, offset in tensor, offset in the masters, length, round)
        self.pieces = []
        for k, lo, hi in self.chunks:
            for i, t_off, c_off, n in shard_pieces(self.sizes, lo, hi):
                self.pieces.append((i, t_off, k * self.cs + c_off, n, k))
        self.master = torch.zeros(self.rounds * self.cs, dtype=torch.float32, device=self.device)
        for i, t_off, s_off, n, _ in self.pieces:
            src = params[i].detach().reshape(-1)[t_off:t_off + n]
            self.master[s_off:s_off + n].copy_(src.to(self.device, torch.float32))
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self._peer = None
        n_flat = self.rounds * self.world * self.cs
        if self.peer_writes:
            self._peer = PeerBuffer(2 * n_flat + 16, self.device, process_group)
            self.flat_weights = self._peer.tensor.view(torch.int16)[:n_flat].view(low_precision)
            self.flat_weights.zero_()
            self._done = torch.zeros(1, dtype=torch.float32, device=self.device)
        else:
            self.flat_weights = torch.zeros(n_flat, dtype=low_precision, device=self.device)
        off = 0
        self.weights = []
        for shape, n in zip(self.shapes, self.sizes):
            self.weights.append(self.flat_weights[off:off + n].view(shape))
            off += n
        for k, lo, hi in self.chunks:  # this rank's chunks start out as the initial weights
            if hi > lo:
                self.flat_weights[lo:hi].copy_(self.master[k * self.cs:k * self.cs + hi - lo])
        for k in range(self.rounds if self.world > 1 else 0):  # every rank starts from the full weights
            self._gather(k).wait()
        self.backend = (backend if backend is not None else
                        CudaZeroBackend(self.device, reserve_sms if self.world > 1 else 0))
        self._keys = [object() for _ in self.pieces]  # one clock slot per piece
        self._planned = False

    def _want_peers(self, peer_writes, backend):
        """Fused update + all-gather (kernel 1 stores the low-precision copies
        into every rank's buffer over NVLink) when the ranks share a node."""
        if peer_writes is not True and peer_writes is not False and peer_writes != "auto":
            raise ValueError("peer_writes must be True, False or 'auto'")
        if self.world == 1 or backend is not None or self.low_precision not in (torch.bfloat16, torch.float16):
            if peer_writes is True:
                raise ValueError("peer writes need several ranks, the CUDA backend and a 16-bit copy")
            return False
        if peer_writes != "auto":
            return peer_writes
        import socket
        hosts = [None] * self.world
        dist.all_gather_object(hosts, socket.gethostname(), group=self.group)
        return len(set(hosts)) == 1 and self.world - 1 <= 15

    def close(self):
        """Release the peer-mapped buffer (collective: every rank calls it).
        ``flat_weights`` and ``weights`` become private copies; views taken from
        them before the call are invalid afterwards."""
        if self._peer is not None:
            self.flat_weights = self.flat_weights.clone()
            self.weights = [w.clone() for w in self.weights]
            self._peer.close()
            self._peer = None

    def _own(self, k):
        base = (k * self.world + self.rank) * self.cs
        return self.flat_weights[base:base + self.cs]

    def _gather(self, k):
        block = self.flat_weights[k * self.world * self.cs:(k + 1) * self.world * self.cs]
        return dist.all_gather_into_tensor(block, self._own(k), group=self.group, async_op=True)

    def _fin_flags(self):
        flags = _lib.MB_FIN_GATE if self.gate else 0
        if self.max_norm is not None:
            flags |= _lib.MB_FIN_CLIP_TORCH if self.clip_mode == "torch" else _lib.MB_FIN_CLIP_DISK
        return flags

    @torch.no_grad()
    def step(self, grads, events=None) -> None:
        """One step with the full, already reduced gradients (one tensor per
        parameter, same shapes; FP32, FP16 or BF16, one dtype). ``events``
        (optional, 4 CUDA events) are recorded on the current stream before
        the statistics, after the finalize, after the last update round and
        after the last all-gather."""
        self.begin(grads, events=events)
        self.finish(events=events)

    @torch.no_grad()
    def begin(self, grads, events=None, record=None) -> None:
        """The first half of ``step``: the plan, the statistics, their all-reduce
        and the finalize (skip, clip and clocks decided on the device). With
        ``record`` (2 FP64 on this device: a caller's {sum of squares,
        nonfinite}, already summed over every rank and covering these
        gradients), the finalize decides from it instead, with no statistics
        pass and no all-reduce here, so one decision covers a larger step
        (ZeroHybridMuonAdamW). ``finish`` must follow on every rank."""
        grads = list(grads)
        if len(grads) != len(self.sizes):
            raise ValueError("one gradient per parameter expected")
        gdt = grads[0].dtype
        if any(g.dtype != gdt for g in grads):
            raise ValueError("all gradients must share a dtype")
        flat = [g.reshape(-1) for g in grads]
        entries, rounds = [], []
        for i, t_off, s_off, n, k in self.pieces:
            g = flat[i][t_off:t_off + n]
            if g.device != self.device or not g.is_contiguous():
                raise ValueError("gradients must be contiguous and on the optimizer's device")
            own = self._own(k)
            c_off = s_off - k * self.cs
            entries.append((self.master[s_off:s_off + n], self.exp_avg[s_off:s_off + n],
                            self.exp_avg_sq[s_off:s_off + n], g, own[c_off:c_off + n], 0))
            rounds.append(k)
        if events:
            events[0].record()
        self._planned = bool(entries)
        if entries:
            self.backend.prepare(self._keys, entries, rounds, self.lr, self.betas, self.eps, self.weight_decay,
                                 gdt, self.low_precision)
            if record is None:
                self.backend.stats(self._fin_flags(), self.max_norm)
            else:
                self.backend.finalize_opts(self._fin_flags(), self.max_norm)
        if record is not None:
            if entries:
                self.backend.record().copy_(record)
        else:
            if not entries:
                self.backend.record().zero_()
            if self.world > 1:
                dist.all_reduce(self.backend.record(), group=self.group)
        if entries:
            self.backend.finalize()
        if events:
            events[1].record()

    @torch.no_grad()
    def finish(self, events=None) -> None:
        """The second half of ``step``: the update rounds (each launch first reads
        the skip flag) and the all-gather of the low-precision weights."""
        works = []
        deltas = self._peer.deltas if self._peer is not None else None
        for k in range(self.rounds):
            if self._planned:
                self.backend.apply_round(k, deltas) if deltas else self.backend.apply_round(k)
            if self.world > 1 and deltas is None:
                works.append(self._gather(k))
        if events:
            events[2].record()
        for w in works:
            w.wait()
        if deltas is not None:
            # every rank's stores into every buffer are complete once all ranks pass this
            dist.all_reduce(self._done, group=self.group)
        if events:
            events[3].record()
        if self.sync:
            self.check()

    def skip_flag(self):
        """The backend's handle on this step's device skip flag (set by
        ``begin``), or None when this rank holds no piece of the group."""
        return self.backend.skip_flag() if self._planned else None

    def record(self) -> torch.Tensor:
        """The step's all-reduced {sum of squares, nonfinite} record."""
        return self.backend.record()

    def check(self) -> None:
        """Wait for the last step and raise FloatingPointError if it was refused."""
        info = self.backend.last_step()
        if info["status"]:
            _lib.check(info["status"], "optimizer not updated")

    def last_step(self) -> dict:
        return self.backend.last_step()

    def state_dict(self) -> dict:
        """This rank's chunks: masters, moments, layout and hyperparameters."""
        return dict(rank=self.rank, world=self.world, rounds=self.rounds, chunk=self.cs, chunks=self.chunks,
                    master=self.master.cpu(), exp_avg=self.exp_avg.cpu(), exp_avg_sq=self.exp_avg_sq.cpu(),
                    lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.weight_decay)


# ----------------------------------------------------- Hybrid Muon + AdamW ----

def deal_matrices(shapes, world, rank_batches):
    """Whole-matrix sharding of the Muon group.

    shapes: the Muon matrices' shapes in order. Matrices of one shape are dealt
    round-robin over the ranks (one shape = one Newton-Schulz cost, so every rank
    gets the same FLOPs up to one matrix per shape). ``rank_batches(count, rows,
    cols)`` gives the batch sizes one rank uses for ``count`` matrices of a shape.
    Returns the rounds: a list of {rank: [matrix index, ...]}; in every round each
    rank steps one batch of one shape, so the rounds line up across ranks."""
    groups = {}
    for i, s in enumerate(shapes):
        groups.setdefault(tuple(s), []).append(i)
    rounds = []
    for shape, idx in groups.items():
        per_rank = [idx[r::world] for r in range(world)]
        sizes = rank_batches(len(per_rank[0]), *shape)  # rank 0 holds the most
        b = 0
        for size in sizes:
            rounds.append({r: per_rank[r][b:b + size] for r in range(world)})
            b += size
    return rounds


class CudaHybridBackend:
    """Kernel calls of one sharded Hybrid step on the rank's GPU (C-ABI library)."""

    def __init__(self, device, ns_dtype="auto", max_sms=0):
        self.device = torch.device(device)
        self.engine = StepEngine(self.device)
        self.ns_dtype = ns_dtype
        self.max_sms = int(max_sms)  # the Muon GEMMs' SM cap (0: all): the rest run the all-gathers
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._keys = {}
        self._plan = None
        self._fin = self.engine.finalize_opts(_lib.MB_FIN_GATE, None)

    def gate_record(self, grads) -> torch.Tensor:
        """Kernel 2 over ``grads``: the {sumsq, nonfinite} record (2 x FP64 on the device)."""
        rec = self.engine.state_buf[:16].view(torch.float64)
        if not grads:
            rec.zero_()
            return rec
        gdt = grads[0].dtype
        flat = [g.reshape(-1) for g in grads]
        keys = self._keys.get(len(flat))  # clock slots are unused by the statistics; reuse them
        if keys is None:
            keys = self._keys[len(flat)] = [object() for _ in flat]
            for k in keys:
                self.engine.slot(k, 0)
        entries = [(g, g, g, g, None, 0) for g in flat]
        plan = self.engine.prepare(entries, [(0.0, .9, .9, 1e-8, 0.0, "torch")], _lib.dtype_code(gdt), _lib.MB_NONE,
                                   keys=keys)
        with torch.cuda.device(self.device):
            _lib.check(self.engine.lib.mb_grad_stats(ctypes.byref(plan), None, _lib.stream_handle()), "mb_grad_stats")
        self._plan = plan
        return rec

    def gate_finalize(self, record):
        """The finiteness gate (optimizer.py:50-51) decided on the device from
        ``record`` (the all-reduced {sumsq, nonfinite}): returns the device
        address of the skip flag every Muon launch reads, or None when this
        rank has computed no statistics yet (it then launches no Muon kernel)."""
        if self._plan is None:
            return None
        rec = self.engine.state_buf[:16].view(torch.float64)
        if rec.data_ptr() != record.data_ptr():
            rec.copy_(record)
        with torch.cuda.device(self.device):
            _lib.check(self.engine.lib.mb_step_finalize(ctypes.byref(self._plan), ctypes.byref(self._fin),
                                                        _lib.stream_handle()), "mb_step_finalize")
        return self.engine.state_buf.data_ptr() + _lib.StepState.skip.offset

    def muon_batch(self, params, moms, grads, outs, lr, weight_decay, skip=None):
        """One kernel-4 step over a batch; ``skip``: device address of a skip flag."""
        from .muon import muon_step_batched
        muon_step_batched(params, moms, grads, outs, lr, weight_decay, self.ns_dtype, self.err, skip, self.max_sms)

    def check_errors(self):
        """Raise RuntimeError if a bounded wait of a Muon launch expired (waits for the stream)."""
        if int(self.err.item()):
            self.err.zero_()
            raise RuntimeError("muon step: a bounded wait expired on the device")


class ZeroHybridMuonAdamW:
    """HybridMuonAdamW (streamtrain/optimizer.py:34-70) sharded over the GPUs of
    one node, one process per GPU.

    The Muon matrices are sharded whole (Newton-Schulz needs the full matrix):
    ``deal_matrices`` gives each rank the same number of matrices of each shape.
    Rank r keeps the FP32 masters and momentum of its matrices; the AdamW group
    (embedding, norms, biases) is a ``ZeroAdamW`` over the flat space. Every rank
    holds the full low-precision weights (``weights``, one tensor per parameter
    in ``params`` order). One step, enqueued without a host read:

      1. kernel 2 (finiteness) over this rank's Muon gradients and its AdamW
         chunks; all_reduce of the 16-byte record; the one-block finalize
         decides the gate on the device (optimizer.py:50-51);
      2. per round: this rank's batch of one shape through kernel 4 (every
         launch reads the skip flag first), writing the BF16 copies into place,
         then all_gather_into_tensor of the round's block (in place, on NCCL's
         stream) while the next round computes;
      3. the AdamW group's ZeRO-1 step, finalized from the same record (no
         second statistics pass or all-reduce; kernel 1 and its all-gathers).

    ``reserve_sms`` (with several ranks) caps the Muon GEMMs at SMs -
    reserve_sms, leaving SMs to NCCL's round all-gathers; 0 (the default, the
    faster setting measured at N=2) gives the GEMMs every SM.

    A refused step changes nothing on any rank (the all-gathers carry the
    unchanged weights). With ``sync=True`` (the default, the reference's
    behaviour) ``step`` then raises FloatingPointError on every rank; with
    ``sync=False`` it only enqueues and ``check()`` raises later.

    ``params`` are the model's parameters; ``muon`` selects the Muon ones
    (default: ``partition(model)`` when ``model`` is given)."""

    def __init__(self, model=None, lr=1e-3, muon_lr=None, weight_decay=.01, *, params=None, muon=None,
                 low_precision=torch.bfloat16, process_group=None, device=None, backend=None, adam_backend=None,
                 ns_dtype="auto", workspace_limit=4 << 30, adam_rounds=4, sync=True, reserve_sms=0):
        from .muon import batch_plan, partition
        if model is not None:
            muon_list, adam_list = partition(model)
            params = list(model.parameters())
        else:
            params = list(params)
            ids = {id(p) for p in (muon or [])}
            muon_list = [p for p in params if id(p) in ids]
            adam_list = [p for p in params if id(p) not in ids]
        if not params:
            raise ValueError("ZeroHybridMuonAdamW needs parameters")
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else params[0].device
        self.lr = lr if muon_lr is None else muon_lr
        self.weight_decay = weight_decay
        self.low_precision = low_precision
        self.sync = bool(sync)
        self.params = params
        self.muon = muon_list
        self.adam_params = adam_list
        for p in self.muon:
            if p.dim() != 2:
                raise ValueError("Muon parameters must be 2-D")
        if backend is None:
            # with several ranks the Muon GEMMs may leave reserve_sms SMs to NCCL's round all-gathers
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            cap = max(2, sms - int(reserve_sms)) if self.world > 1 and reserve_sms else 0
            self.backend = CudaHybridBackend(self.device, ns_dtype, cap)
            plan = lambda n, r, c: batch_plan(n, r, c, workspace_limit)  # noqa: E731
        else:
            self.backend = backend
            plan = getattr(backend, "batch_plan", lambda n, r, c: [n] if n else [])
        self.rounds = deal_matrices([tuple(p.shape) for p in self.muon], self.world, plan)
        # flat low-precision buffer of the Muon group: per round, one equal block per rank
        self.layout = {}  # muon index -> (round, offset in the flat buffer)
        self.round_blocks = []  # (offset, block elements per rank)
        off = 0
        for k, rd in enumerate(self.rounds):
            per = max(sum(self.muon[i].numel() for i in rd[r]) for r in range(self.world))
            per = -(-per // ALIGN) * ALIGN
            for r in range(self.world):
                o = off + r * per
                for i in rd[r]:
                    self.layout[i] = (k, o)
                    o += self.muon[i].numel()
            self.round_blocks.append((off, per))
            off += per * self.world
        self.flat_muon = torch.zeros(max(off, 1), dtype=low_precision, device=self.device)
        self.muon_weights = [self.flat_muon[o:o + p.numel()].view(p.shape)
                             for p, (_, o) in ((self.muon[i], self.layout[i]) for i in range(len(self.muon)))]
        self.owned = [i for rd in self.rounds for i in rd[self.rank]]
        self.master = {i: self.muon[i].detach().to(self.device, torch.float32).clone() for i in self.owned}
        self.momentum = {}
        self._new_momentum = []
        self._record = torch.zeros(2, dtype=torch.float64, device=self.device)
        for i in range(len(self.muon)):  # every rank starts from the full weights
            self.muon_weights[i].copy_(self.muon[i].detach().to(self.device))
        # the AdamW group finalizes from the gate's all-reduced record (gate on, no host read)
        self.adam = ZeroAdamW(adam_list, lr=lr, betas=(.9, .95), eps=1e-8, weight_decay=weight_decay, gate=True,
                              sync=False, low_precision=low_precision, process_group=process_group,
                              device=self.device, backend=adam_backend, rounds=adam_rounds) if adam_list else None
        index = {id(p): i for i, p in enumerate(self.muon)}
        aindex = {id(p): i for i, p in enumerate(adam_list)}
        self.weights = [self.muon_weights[index[id(p)]] if id(p) in index else self.adam.weights[aindex[id(p)]]
                        for p in params]

    def _gather(self, k):
        off, per = self.round_blocks[k]
        block = self.flat_muon[off:off + per * self.world]
        own = block[self.rank * per:(self.rank + 1) * per]
        return dist.all_gather_into_tensor(block, own, group=self.group, async_op=True)

    @torch.no_grad()
    def step(self, grads=None) -> None:
        """One step. ``grads``: the full, already reduced gradients in ``params``
        order (default: each parameter's ``.grad``); Muon gradients of one shape
        share a dtype."""
        grads = [p.grad for p in self.params] if grads is None else list(grads)
        if len(grads) != len(self.params):
            raise ValueError("one gradient per parameter expected")
        gmap = {id(p): g for p, g in zip(self.params, grads)}
        muon_grads = [gmap[id(p)] for p in self.muon]
        adam_grads = [gmap[id(p)] for p in self.adam_params]
        if any(g is None for g in muon_grads + adam_grads):
            raise ValueError("every parameter needs a gradient")
        muon_grads = [g.to(self.device).contiguous() for g in muon_grads]
        # 1. finiteness over this rank's share, one decision on every rank
        own_grads = [muon_grads[i] for i in self.owned]
        if self.adam is not None:
            for i, t_off, _, n, _ in self.adam.pieces:
                own_grads.append(adam_grads[i].reshape(-1)[t_off:t_off + n])
        by_dtype = {}
        for g in own_grads:
            by_dtype.setdefault(g.dtype, []).append(g)
        rec = self._record
        rec.zero_()
        for gs in by_dtype.values():
            rec += self.backend.gate_record(gs)
        if self.world > 1:
            dist.all_reduce(rec, group=self.group)
        skip = self.backend.gate_finalize(rec)
        # 2. Muon rounds, each all-gathered while the next computes
        works = []
        self._new_momentum = []
        for k, rd in enumerate(self.rounds):
            mine = rd[self.rank]
            if mine:
                for i in mine:
                    if i not in self.momentum:
                        self.momentum[i] = torch.zeros_like(self.master[i])
                        self._new_momentum.append(i)
                self.backend.muon_batch([self.master[i] for i in mine], [self.momentum[i] for i in mine],
                                        [muon_grads[i] for i in mine], [self.muon_weights[i] for i in mine],
                                        self.lr, self.weight_decay, skip)
            if self.world > 1:
                works.append(self._gather(k))
        # 3. the AdamW group, finalized from the same record
        if self.adam is not None:
            self.adam.begin(adam_grads, record=rec)
            self.adam.finish()
        for w in works:
            w.wait()
        if self.sync:
            self.check()

    def check(self) -> None:
        """Wait for the last step and raise what it reported: RuntimeError if a
        bounded device wait expired, FloatingPointError if the gate refused the
        step (nothing changed; momentum buffers it created are dropped, as the
        reference never creates them). Every rank reads the same all-reduced
        record, so every rank raises alike."""
        self.backend.check_errors()
        sumsq, bad = (float(x) for x in self._record.cpu())
        if bad >= _lib.TIMEOUT_MARK:
            raise RuntimeError("gradient statistics: a bounded wait expired on the device")
        if bad != 0.0 or not math.isfinite(sumsq):
            for i in self._new_momentum:
                self.momentum.pop(i, None)
            self._new_momentum = []
            raise FloatingPointError('nonfinite gradient; optimizer not updated')
        self._new_momentum = []

    def close(self):
        """Release the AdamW group's peer-mapped buffer (collective)."""
        if self.adam is not None:
            self.adam.close()
            aindex = {id(p): i for i, p in enumerate(self.adam_params)}
            mindex = {id(p): i for i, p in enumerate(self.muon)}
            self.weights = [self.muon_weights[mindex[id(p)]] if id(p) in mindex else self.adam.weights[aindex[id(p)]]
                            for p in self.params]

    def state_dict(self) -> dict:
        """This rank's share: Muon masters and momentum by Muon index, the AdamW shard."""
        return dict(rank=self.rank, world=self.world, lr=self.lr, weight_decay=self.weight_decay,
                    master={i: t.cpu() for i, t in self.master.items()},
                    momentum={i: t.cpu() for i, t in self.momentum.items()},
                    adam=self.adam.state_dict() if self.adam is not None else None)
