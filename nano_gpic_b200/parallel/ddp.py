"""Data parallelism over the flat parameter / gradient buffers: the flat layout (buckets in the order the backward
finishes gradients, owners inside each bucket), gradient collectives overlapped with the backward, and two modes.

  ddp   The reference's DDP (Lightning DDPStrategy with bucket_cap_mb=1000, baselines/PixelGen/configs_h100/
        lite_ladder.yaml:7-12; `gradient_as_bucket_view`): one fp32 all-reduce per bucket. Gradients are pre-scaled by
        1/world in the loss, so the sum is the mean. Every rank holds the full averaged gradient; Muon units are
        orthogonalised by their longest-processing-time owner and the bf16 results all-gathered (MuonAdamW; reference
        baselines/PixelGen/src/optim/muon.py:150-216); AdamW runs replicated.

  zero  Sharded optimizer, the role of the reference's FSDP2 + ShardMuonAdamW (baselines/PixelGen/src/utils/
        fsdp_setup.py:116-148, src/optim/muon_fsdp.py:41-188), laid out for one B200's 180 GB: inside each bucket the
        parameters are placed owner-major. Owners are chosen by longest-processing-time on the Muon cost
        (rows * cols * min(rows, cols)), or numel for AdamW parameters. Each owner's segment is padded to a common
        size, so ONE fp32 reduce-scatter per bucket leaves every owner the summed gradient of WHOLE parameters and
        Muon needs no all-to-all (the reference sends rows to owners and back with two all_to_all_single). The owner
        clips (global norm from one scalar all-reduce), runs Muon / AdamW on its parameters with its own optimizer
        state, writes them in bf16, and ONE bf16 all-gather per bucket refreshes every rank's compute weights.
        Other owners' fp32 masters and optimizer state are gathered only when a checkpoint needs them.
        Per optimizer step and rank this moves (world-1)/world of the fp32 gradients once (reduce-scatter) and of the
        bf16 weights once (all-gather): less than DDP's all-reduce + Muon all-gather, and less than FSDP2 + two
        all-to-alls.

Transport (zero mode): "nccl" (reduce_scatter_tensor / all_gather_into_tensor per bucket, the baseline) or "p2p"
(P2PTransport below: this package's kernels over CUDA-IPC peer memory: each rank pushes its gradient segments into
the owners' receive slots with NVLink stores and epoch flags, the owner sums them in rank order together with the
sum of squares for the clip, and after the update each owner writes its bf16 weights straight into every rank's
compute-weight buffer; csrc/p2p.cu).

Overlap: the model calls `hook(n)` at the start of each block's backward on the LAST micro-batch, meaning the first n
backward stages (final layer, image blocks from the last, text blocks from the last) hold final gradients; every
bucket made only of finished stages is reduced at once on a side CUDA stream, under the rest of the backward.
"""
import torch
import torch.distributed as dist

from ..ops.optim import scale_
from .flat import FlatParams, _round


# ------------------------------------------------------------------------------------------------------- layout
def backward_stages(model):
    """Lists of trainable parameters in the order the backward finishes their gradients. For JiT_T2I: final layer,
    image blocks last to first, text blocks last to first, then everything else (embedders, time MLP, caption
    table). Other modules: one stage."""
    seen, stages = set(), []

    def add(mod_or_params):
        ps = [p for p in (mod_or_params.parameters() if hasattr(mod_or_params, "parameters") else mod_or_params)
              if p.requires_grad and id(p) not in seen]
        seen.update(id(p) for p in ps)
        stages.append(ps)

    if hasattr(model, "blocks") and hasattr(model, "final_layer"):
        add(model.final_layer)
        for blk in reversed(model.blocks):
            add(blk)
        for blk in reversed(getattr(model, "text_refine_blocks", [])):
            add(blk)
    add([p for p in model.parameters()])
    return stages


class Bucket:
    def __init__(self, start, end, seg, last_stage, params, replicated=False):
        self.start, self.end, self.seg = start, end, seg  # [start, end) of the flat buffers; owner segment size
        self.last_stage = last_stage  # ready once stages [0, last_stage] are finished
        self.params = params
        self.replicated = replicated  # all-reduced and updated on every rank (ddp mode, zero mode's fp32 consumers)


def replicated_in_zero(p):
    """Parameters the forward reads in fp32 (vectors: norm weights, biases; and those marked `_replicate`) stay
    replicated in zero mode, as the reference's FSDP2 keeps RMSNorm weights replicated (fsdp_setup.py:21-26,
    271-280): their gradients are all-reduced and every rank updates them."""
    return p.ndim < 2 or getattr(p, "_replicate", False)


class Layout:
    """Flat order, offsets and buckets for `world` ranks. mode "ddp": parameters in backward order; "zero": owner-major
    inside each bucket with equal (padded) owner segments."""

    def __init__(self, model, world, mode="ddp", bucket_numel=250_000_000):
        assert mode in ("ddp", "zero"), mode
        self.world, self.mode = world, mode
        stages = backward_stages(model)
        self.params, self.offsets, self.buckets, self.owner = [], [], [], {}
        groups, cur, cur_n = [], [], 0
        for si, ps in enumerate(stages):
            cur += [(si, p) for p in ps]
            cur_n += sum(p.numel() for p in ps)
            if cur_n >= bucket_numel:
                groups.append(cur)
                cur, cur_n = [], 0
        if cur:
            groups.append(cur)
        off = 0
        rep = []
        for g in groups:
            last = max(si for si, _ in g)
            ps = [p for _, p in g]
            if mode == "zero" and world > 1:
                rep += [p for p in ps if replicated_in_zero(p)]
                ps = [p for p in ps if not replicated_in_zero(p)]
                if not ps:
                    continue
            start = off
            if mode == "ddp" or world == 1:
                for p in ps:
                    self.params.append(p)
                    self.offsets.append(off)
                    self.owner[id(p)] = None
                    off = _round(off + p.numel())
                seg = off - start
            else:
                load = [0] * world
                mine = [[] for _ in range(world)]
                order = sorted(range(len(ps)), key=lambda i: (-self.cost(ps[i]), i))
                for i in order:
                    r = min(range(world), key=lambda q: (load[q], q))
                    mine[r].append(i)
                    load[r] += _round(ps[i].numel())
                seg = _round(max(load))
                for r in range(world):
                    o = start + r * seg
                    for p in (ps[i] for i in sorted(mine[r])):
                        self.params.append(p)
                        self.offsets.append(o)
                        self.owner[id(p)] = r
                        o = _round(o + p.numel())
                off = start + world * seg
            self.buckets.append(Bucket(start, off, seg, last, ps))
        if rep:
            start = off
            for p in rep:
                self.params.append(p)
                self.offsets.append(off)
                self.owner[id(p)] = None
                off = _round(off + p.numel())
            self.buckets.append(Bucket(start, off, off - start, len(stages) - 1, rep, replicated=True))
        self.numel = off

    @staticmethod
    def cost(p):
        if getattr(p, "_muon_parts", None):
            rows, cols = p.shape[0] // p._muon_parts, p.shape[1]
            return p._muon_parts * rows * cols * min(rows, cols)
        return p.numel()

    def flat(self, model, device=None):
        return FlatParams(model, device=device, params=self.params, offsets=self.offsets, numel=self.numel)

    def padding(self):
        used = sum(_round(p.numel()) for p in self.params)
        return 1.0 - used / max(self.numel, 1)


# ---------------------------------------------------------------------------------------------- collectives
def _gloo(group):
    return dist.get_backend(group) == "gloo"


def _reduce_scatter_inplace(buf, seg, rank, group):
    """Sum over ranks; rank r's segment [r*seg, (r+1)*seg) receives its sums (NCCL in-place reduce-scatter)."""
    if _gloo(group):  # gloo has no reduce-scatter: the same sums through an all-reduce
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    else:
        dist.reduce_scatter_tensor(buf[rank * seg:(rank + 1) * seg], buf, op=dist.ReduceOp.SUM, group=group)


def _all_gather_inplace(buf, seg, rank, world, group):
    """Every rank's segment r of buf from rank r (NCCL in-place all-gather)."""
    if _gloo(group):
        parts = list(buf.view(world, seg).unbind(0))
        dist.all_gather(parts, buf[rank * seg:(rank + 1) * seg].clone(), group=group)
    else:
        dist.all_gather_into_tensor(buf, buf[rank * seg:(rank + 1) * seg], group=group)


class P2PTransport:
    """Peer buffers of one node for zero mode: the flat gradient (fp32), a receive buffer of the same size, the bf16
    compute weights, and int64 [W][nb] flag / acknowledgement arrays, all cudaMalloc'd and opened by every rank through
    CUDA IPC. Collective setup (every rank constructs it)."""

    MAX_PARTIALS = 512  # sum-of-squares partials per bucket (bounds the reduce kernel's grid)

    def __init__(self, numel, n_buckets, device, group=None):
        from .._ext import ext
        self.ext = ext()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world <= 8, "peer-memory transport: one node of at most 8 GPUs"
        self.nb = n_buckets
        dev = torch.device(device).index
        W, nb = self.world, n_buckets
        alloc = lambda nbytes: self.ext.p2p_alloc(int(nbytes), dev)
        self.raw = {"grad": alloc(numel * 4), "recv": alloc(numel * 4), "w16": alloc(numel * 2),
                    "flags": alloc(W * nb * 8), "acks": alloc(W * nb * 8), "wflags": alloc(W * nb * 8)}
        self.grad = self.raw["grad"].view(torch.float32)
        self.recv = self.raw["recv"].view(torch.float32)
        self.w16 = self.raw["w16"].view(torch.bfloat16)
        self.flags = self.raw["flags"].view(torch.int64)
        self.acks = self.raw["acks"].view(torch.int64)
        self.wflags = self.raw["wflags"].view(torch.int64)
        # flat optimizer state and Muon output for the fused apply (only this rank's owned ranges are used)
        self.m1 = torch.zeros(numel, dtype=torch.float32, device=device)
        self.m2 = torch.zeros(numel, dtype=torch.float32, device=device)
        self.upd = torch.zeros(numel, dtype=torch.bfloat16, device=device)
        self.tables = None
        self.counters = torch.zeros(2 * nb + 2, dtype=torch.int32, device=device)
        self.bcast_counter = torch.zeros(2, dtype=torch.int32, device=device)
        self.sumsq = torch.zeros(nb, self.MAX_PARTIALS, dtype=torch.float32, device=device)
        mine = {k: self.ext.p2p_export(v).tolist() for k, v in self.raw.items()}
        every = [None] * W
        dist.all_gather_object(every, mine, group=group)
        self.peer = {}
        self._opened = []
        for k, v in self.raw.items():
            ptrs = []
            for r in range(W):
                if r == self.rank:
                    ptrs.append(v.data_ptr())
                else:
                    p = self.ext.p2p_import(torch.tensor(every[r][k], dtype=torch.uint8), dev)
                    self._opened.append(p)
                    ptrs.append(p)
            self.peer[k] = ptrs
        dist.barrier(group=group)

    def close(self):
        """Collective: unmap the peers' buffers (before any rank frees its own)."""
        torch.cuda.synchronize()
        dist.barrier()
        for p in self._opened:
            self.ext.p2p_close(p)
        self._opened = []
        dist.barrier()

    def reduce_scatter(self, b, start, seg, epoch):
        """Bucket b ([W segments of seg fp32] at start): this rank's segment becomes the sum over ranks."""
        self.sumsq[b].zero_()
        self.ext.p2p_reduce_scatter(self.grad, self.recv, self.peer["recv"], self.flags, self.peer["flags"], self.acks,
                                    self.peer["acks"], self.counters, self.sumsq[b], self.rank, self.nb, b, start,
                                    seg, epoch)

    def broadcast_weights(self, master, b, off, n, epoch):
        self.ext.p2p_bcast_bf16(master, self.peer["w16"], self.peer["wflags"], self.bcast_counter, self.rank, self.nb,
                                b, off, n, epoch)

    CHUNK = 16384

    def build_tables(self, layout, flat, rank, opt):
        """Per sharded bucket, the [off, n | kind << 32, coef] rows of this rank's owned parameters (chunks of at most
        CHUNK elements); registers the deferred mode with the optimizer."""
        import struct
        off_of = {id(p): o for p, o in zip(flat.params, flat.offsets)}
        muon_group = next((g for g in opt.param_groups if g.get("use_muon")), None)
        ids = set()
        self.tables = []
        for b in layout.buckets:
            if b.replicated:
                continue
            rows = []
            for p in b.params:
                if layout.owner[id(p)] != rank:
                    continue
                ids.add(id(p))
                muon = getattr(p, "_muon_parts", None) is not None
                coef = 0.0
                if muon:
                    parts = p._muon_parts if muon_group["split"] else 1
                    coef = opt.update_coef(muon_group, (p.shape[0] // parts, p.shape[1]))
                o0 = off_of[id(p)]
                for c in range(0, p.numel(), self.CHUNK):
                    n = min(self.CHUNK, p.numel() - c)
                    w2 = struct.unpack("<q", struct.pack("<ff", coef, 0.0))[0]
                    rows.append([o0 + c, n | ((1 if muon else 0) << 32), w2])
            t = torch.tensor(rows if rows else [[0, 0, 0]], dtype=torch.int64, device=self.grad.device)
            self.tables.append((t, len(rows)))
        opt.defer = {"ids": ids, "off": off_of, "upd": self.upd, "m1": self.m1, "m2": self.m2}

    def fused_apply(self, i, master, grad, ema_buf, scal, epoch):
        t, n = self.tables[i]
        vals = [scal.get("lr_a", 0.0), scal.get("wd_a", 0.0), scal.get("b1", 0.9), scal.get("b2", 0.95),
                scal.get("eps", 1e-8), scal.get("bc1", 1.0), scal.get("rsqrt_bc2", 1.0), scal.get("lr_m", 0.0),
                scal.get("wd_m", 0.0), scal.get("ema_keep", 1.0)]
        self.ext.p2p_fused_apply(t, n, master, grad, self.m1, self.m2, self.upd, ema_buf, self.peer["w16"],
                                 self.peer["wflags"], self.bcast_counter, [float(v) for v in vals], self.rank, self.nb,
                                 i, epoch)

    def wait_weights(self, b0, b1, epoch):
        self.ext.p2p_wait(self.wflags, self.world, self.rank, self.nb, b0, b1, epoch)


class DataParallel:
    """The gradient / weight synchronisation of one data-parallel group over a Layout's flat buffers."""

    def __init__(self, model, layout, flat, group=None, overlap=True, p2p=None):
        self.model, self.layout, self.flat, self.group = model, layout, flat, group
        self.mode = layout.mode
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world == layout.world
        self.overlap = overlap
        self.cuda = flat.grad.is_cuda
        self.comm = torch.cuda.Stream(device=flat.grad.device) if self.cuda else None
        self._launched = set()
        self.early = 0  # buckets launched under the backward in the last step (overlap statistics)
        self.p2p = p2p  # P2PTransport (zero mode over peer memory) or None (NCCL)
        self.epoch = 0  # optimizer steps synchronised so far (the peer flags' epochs)
        self.opt = None  # with p2p: the optimizer whose owned-parameter update the fused kernel applies
        self.ema_buf = None  # with p2p + fused apply: the EMA's flat buffer (owned ranges updated by the kernel)
        self.ema_keep = 1.0
        # zero mode: the parameters this rank updates (its own and the replicated ones)
        self.owned = None if self.mode == "ddp" else {id(p) for p in layout.params
                                                      if layout.owner[id(p)] in (self.rank, None)}
        # peer-memory transport: its kernels record a timed-out wait in the device status word and skip their work.
        # The word is copied to the host behind each step's weight refresh and read in the next step's finish_grads
        # (by then long complete), so a lost peer stops the run with NanoCommTimeout one step late, with no host
        # synchronisation inside a step. Anything with post() / poll() can stand in (tests).
        self.status = None
        if p2p is not None:
            from ..ops.status import AsyncCheck
            self.status = AsyncCheck()

    @torch.no_grad()
    def after_load(self):
        """After optimizer state was loaded: the fused kernel's flat AdamW state takes the loaded values and the state
        entries become its views again."""
        if self.p2p is None or self.opt is None:
            return
        d = self.opt.defer
        for p, st in self.opt.state.items():
            if id(p) not in d["ids"] or "exp_avg" not in st:
                continue
            o = d["off"][id(p)]
            for k, buf in (("exp_avg", d["m1"]), ("exp_avg_sq", d["m2"])):
                v = buf[o:o + p.numel()]
                v.copy_(st[k].reshape(-1).to(v.device))
                st[k] = v.view(p.shape)
            d["steps"] = int(float(st["step"]))

    def attach_optimizer(self, opt):
        """zero mode over peer memory: the update of the owned parameters (AdamW and the Muon apply) runs in the
        fused kernel together with the weight broadcast."""
        if self.p2p is not None:
            self.opt = opt
            self.p2p.build_tables(self.layout, self.flat, self.rank, opt)

    # ----------------------------------------------------------------------------------------- gradients
    def arm(self):
        """Before the backward of the last micro-batch: reduce buckets as their stages finish."""
        self._launched = set()
        self.epoch += 1
        if self.overlap:
            self.model._bwd_hook = self._stages_done

    def _stages_done(self, n):
        for i, b in enumerate(self.layout.buckets):
            if i not in self._launched and b.last_stage < n:
                self._launch(i)

    def _launch(self, i):
        self._launched.add(i)
        b = self.layout.buckets[i]
        g = self.flat.grad[b.start:b.end]
        if self.cuda:
            self.comm.wait_stream(torch.cuda.current_stream(g.device))
            with torch.cuda.stream(self.comm):
                self._reduce(g, b)
        else:
            self._reduce(g, b)

    def _reduce(self, g, b):
        if self.mode == "ddp" or b.replicated:
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group)
        elif self.p2p is not None:
            self.p2p.reduce_scatter(self.layout.buckets.index(b), b.start, b.seg, self.epoch)
        else:
            _reduce_scatter_inplace(g, b.seg, self.rank, self.group)

    def finish_grads(self):
        """After the backward: reduce what is left and make the compute stream wait for every collective. Raises
        NanoCommTimeout when the previous step's peer-memory kernels recorded a timed-out wait."""
        self.model._bwd_hook = None
        if self.status is not None:
            self.status.poll()
        self.early = len(self._launched)
        for i in range(len(self.layout.buckets)):
            if i not in self._launched:
                self._launch(i)
        if self.cuda:
            torch.cuda.current_stream(self.flat.grad.device).wait_stream(self.comm)

    def _sharded(self):
        return [b for b in self.layout.buckets if not b.replicated]

    def own_slices(self, buf):
        """The parts of a flat buffer this rank is responsible for: all of it in ddp mode; its owner segments (and
        the replicated bucket, which every rank holds) in zero mode."""
        if self.mode == "ddp":
            return [buf]
        return ([buf[b.start + self.rank * b.seg:b.start + (self.rank + 1) * b.seg] for b in self._sharded()] +
                [buf[b.start:b.end] for b in self.layout.buckets if b.replicated])

    @torch.no_grad()
    def grad_norm(self):
        """Global 2-norm of the (reduced) gradient: local sum of squares of the owned segments, one scalar
        all-reduce, plus the replicated part (identical on every rank, counted once)."""
        if self.mode == "ddp":
            return self.flat.grad.norm()
        g = self.flat.grad
        z = torch.zeros((), device=g.device)
        if self.p2p is not None:  # the reduce kernels left per-CTA partial sums of squares (fixed order: deterministic)
            sq = self.p2p.sumsq.sum()
        else:
            sq = sum((s.pow(2).sum() for s in (g[b.start + self.rank * b.seg:b.start + (self.rank + 1) * b.seg]
                                               for b in self._sharded())), z)
        dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=self.group)
        sq = sq + sum((g[b.start:b.end].pow(2).sum() for b in self.layout.buckets if b.replicated), z)
        return sq.sqrt()

    @torch.no_grad()
    def scale_grads(self, coef):
        for s in self.own_slices(self.flat.grad):
            scale_(s, coef)

    # ------------------------------------------------------------------------------------------- weights
    @torch.no_grad()
    def refresh_weights(self):
        """After the optimizer step: the bf16 compute weights of every rank from the owners' fp32 masters."""
        if self.mode == "ddp":
            self.flat.sync_bf16()
            return
        for i, b in enumerate(self.layout.buckets):
            if b.replicated:
                self.flat.data16[b.start:b.end].copy_(self.flat.data[b.start:b.end])
                continue
            lo = b.start + self.rank * b.seg
            if self.p2p is not None and self.opt is not None:  # update + EMA + bf16 to every rank, then flags
                scal = dict(self.opt.deferred or {}, ema_keep=self.ema_keep)
                self.p2p.fused_apply(i, self.flat.data, self.flat.grad, self.ema_buf, scal, self.epoch)
                continue
            if self.p2p is not None:  # owner -> bf16 into every rank's weights, then flags
                self.p2p.broadcast_weights(self.flat.data, i, lo, b.seg, self.epoch)
                continue
            self.flat.data16[lo:lo + b.seg].copy_(self.flat.data[lo:lo + b.seg])
            _all_gather_inplace(self.flat.data16[b.start:b.end], b.seg, self.rank, self.world, self.group)
        if self.p2p is not None:  # the next forward reads every owner's weights: wait (on the compute stream) for the
            # sharded buckets' flags (they come first; the replicated bucket was refreshed locally above)
            self.p2p.wait_weights(0, len(self._sharded()), self.epoch)
        if self.status is not None:
            self.status.post()

    def own_ranges(self):
        """[start, end) ranges of the flat buffers this rank keeps current (None in ddp mode: all of them)."""
        if self.mode == "ddp":
            return None
        return ([(b.start + self.rank * b.seg, b.start + (self.rank + 1) * b.seg) for b in self._sharded()] +
                [(b.start, b.end) for b in self.layout.buckets if b.replicated])

    @torch.no_grad()
    def gather_flat(self, buf):
        """zero mode: every owner segment of a flat-layout buffer (fp32 masters, the EMA) from its owner."""
        if self.mode == "ddp":
            return
        for b in self._sharded():
            _all_gather_inplace(buf[b.start:b.end], b.seg, self.rank, self.world, self.group)

    def gather_master(self):
        """zero mode: every rank's fp32 masters from their owners (for checkpoints)."""
        self.gather_flat(self.flat.data)

    def prepare_checkpoint(self, opt, ema=None, full=True):
        """Collective (every rank calls it): the full fp32 weights, EMA and (full=True) optimizer state on every rank,
        so the checkpoint builder sees the unsharded state."""
        if self.mode == "ddp":
            return
        self.gather_master()
        if ema is not None and ema.buf is not None:
            ema.join()
            self.gather_flat(ema.buf)
        if full:
            self.gather_optimizer_state(opt)

    @torch.no_grad()
    def gather_optimizer_state(self, opt):
        """zero mode: every rank's optimizer state for every parameter from its owner, through flat buffers of the
        layout (one all-gather per bucket and state kind). Afterwards opt.state_dict() is the full state."""
        if self.mode == "ddp":
            return
        dev = self.flat.data.device
        kinds = {}
        index = {id(p): i for i, p in enumerate(self.flat.params)}
        for grp in opt.param_groups:
            for p in grp["params"]:
                if id(p) not in index:  # frozen parameters have no state
                    continue
                keys = ("momentum_buffer",) if grp.get("use_muon") else ("exp_avg", "exp_avg_sq")
                for k in keys:
                    kinds.setdefault(k, []).append(p)
        for k, ps in kinds.items():
            buf = torch.zeros(self.flat.numel, dtype=torch.float32, device=dev)
            for p in ps:
                st = opt.state.get(p, {})
                if id(p) in self.owned and k in st:
                    o = self.flat.offsets[index[id(p)]]
                    buf[o:o + p.numel()].copy_(st[k].reshape(-1))
            for b in self._sharded():
                _all_gather_inplace(buf[b.start:b.end], b.seg, self.rank, self.world, self.group)
            for p in ps:
                o = self.flat.offsets[index[id(p)]]
                opt.state[p][k] = buf[o:o + p.numel()].view(p.shape).clone()
        steps = [opt.state[p]["step"] for p in kinds.get("exp_avg", []) if "step" in opt.state[p]
                 and id(p) in self.owned]
        s = torch.tensor(float(steps[0]) if steps else 0.0, device=dev)
        dist.all_reduce(s, op=dist.ReduceOp.MAX, group=self.group)
        for p in kinds.get("exp_avg", []):
            old = opt.state[p].get("step")
            opt.state[p]["step"] = s.clone().to(old.device if old is not None else dev)

    @torch.no_grad()
    def broadcast_params(self, src=0):
        dist.broadcast(self.flat.data, src, group=self.group)
        self.flat.sync_bf16()


def make_data_parallel(model, world, mode="ddp", bucket_mb=1000, device=None, group=None, overlap=True,
                       transport="nccl"):
    """Layout + flat buffers + DataParallel for `model` (Muon tags must already be set). bucket_mb counts fp32
    gradient bytes, as the reference's bucket_cap_mb. transport "p2p" (zero mode, CUDA, one node): this package's
    peer-memory kernels instead of NCCL for the reduce-scatter and the weight all-gather."""
    layout = Layout(model, world, mode, bucket_numel=bucket_mb * 1024 * 1024 // 4)
    p2p = None
    if world > 1 and mode == "zero" and transport == "p2p":
        p2p = P2PTransport(layout.numel, len(layout.buckets), device, group=group)
        flat = FlatParams(model, device=device, params=layout.params, offsets=layout.offsets, numel=layout.numel,
                          grad_buf=p2p.grad, data16_buf=p2p.w16)
    else:
        flat = layout.flat(model, device=device)
    dp = DataParallel(model, layout, flat, group=group, overlap=overlap, p2p=p2p) if world > 1 else None
    return layout, flat, dp


# the name the trainer used before the layout existed
GradReducer = DataParallel
