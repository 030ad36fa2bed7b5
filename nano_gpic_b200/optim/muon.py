"""Muon for the hidden matrices of the transformer blocks, AdamW for every other parameter.

Same constructor, param groups, state names (momentum_buffer; step/exp_avg/exp_avg_sq) and update rules as the
reference's MuonAdamW (baselines/PixelGen/src/optim/muon.py:102-254), so optimizer checkpoints are interchangeable:
    m <- beta m + (1 - beta) g                  (beta = 0.95)
    u <- (1 - beta) g + beta m                  (Nesterov)
    O <- msign(u)                               5 quintic Newton-Schulz steps in bf16, coefficients (3.4445, -4.7750,
                                                2.0315), Frobenius normalisation + 1e-7, transposed when tall
    W <- (1 - lr wd) W - lr * coef * O          coef = sqrt(rows / cols) ("mup") or 0.2 sqrt(max) ("moonlight")
With split=True each fused matrix is cut along d_out into its parts (q,k,v; k,v; gate,up; the six adaLN vectors) and
each part ("unit") is orthogonalised on its own (tag_muon_params, reference muon.py:43-61).

Newton-Schulz runs on the tcgen05 GEMM (nano_gpic_b200.ops.gemm.bmm_axpby), batched per unit shape, each step three
GEMMs with the scalings fused in the epilogue: A = X X^T, B = b A + c A A, X = a X + B X (the reference's lever NS,
muon.py:64-86). Units are owned by ranks with the reference's longest-processing-time plan (muon.py:150-175); with one
rank every unit is local. The distributed exchange lives in nano_gpic_b200.parallel.muon_dist.
"""
import math

import torch
import torch.distributed as dist

from ..ops import gemm as G
from ..ops import optim as OPT

NS_COEFFS = (3.4445, -4.7750, 2.0315)
FUSED_PARTS = {"attn.qkv_x.weight": 3, "attn.qkv.weight": 3, "attn.kv_y.weight": 2, "mlp.w12.weight": 2,
               "adaLN_modulation.0.weight": 6}


def tag_muon_params(model, prefixes=("blocks.", "text_refine_blocks.")):
    """Mark the 2-D weights inside the transformer blocks for Muon (p._muon_parts = fused parts along d_out).
    Returns (n_tagged, numel_tagged)."""
    n = numel = 0
    for name, p in model.named_parameters():
        if p.ndim != 2 or not p.requires_grad or not name.startswith(prefixes):
            continue
        parts = next((k for suffix, k in FUSED_PARTS.items() if name.endswith(suffix)), 1)
        assert p.shape[0] % parts == 0, (name, tuple(p.shape), parts)
        p._muon_parts = parts
        p._muon_name = name
        n += 1
        numel += p.numel()
    return n, numel


@torch.no_grad()
def msign(Gm, steps=5, dtype=torch.bfloat16, fused=True):
    """Orthogonalise each matrix of Gm [..., a, b] with the quintic Newton-Schulz iteration. bf16 CUDA inputs run on
    the tcgen05 GEMM with fused alpha/beta epilogues; other dtypes/devices use torch (the fp32 path is the exact
    reference for tests)."""
    a, b, c = NS_COEFFS
    tall = Gm.size(-2) > Gm.size(-1)
    if Gm.is_cuda and dtype == torch.bfloat16 and fused:
        # the normalisation (and, for tall matrices, the transpose) in two passes of this package's kernels, the
        # iteration on the tcgen05 GEMM, the transpose back in one tiled pass: no PyTorch elementwise passes
        squeeze = Gm.dim() == 2
        X = Gm.to(dtype)
        X = (X.unsqueeze(0) if squeeze else X).contiguous()
        X = OPT.ns_normalize(X, transpose=tall)
        for _ in range(steps):
            A = G.bmm_axpby(X, X, False)                       # X X^T
            B = G.bmm_axpby(A, A, False, alpha=c, beta=b, C=A)  # b A + c A A  (A symmetric)
            X = G.bmm_axpby(B, X, True, alpha=1.0, beta=a, C=X)  # a X + B X
        if tall:
            X = OPT.transpose_bf16(X)
        return X[0] if squeeze else X
    X = Gm.to(dtype)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    return X.mT if tall else X


class MuonAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, muon_lr=None,
                 muon_weight_decay=None, muon_momentum=0.95, muon_nesterov=True, ns_steps=5, split=False,
                 fused_adamw=True, ns_dtype="bfloat16", update_scale="mup"):
        assert update_scale in ("mup", "moonlight"), update_scale
        groups = list(params)
        if groups and not isinstance(groups[0], dict):
            groups = [{"params": groups}]
        adam_groups, muon_params = [], []
        for g in groups:
            ps = list(g["params"])
            muon_params += [p for p in ps if hasattr(p, "_muon_parts")]
            rest = [p for p in ps if not hasattr(p, "_muon_parts")]
            if rest:
                adam_groups.append({**g, "params": rest, "use_muon": False, "fused": fused_adamw})
        all_groups = adam_groups
        if muon_params:
            all_groups = all_groups + [{
                "params": muon_params, "use_muon": True,
                "lr": muon_lr if muon_lr is not None else lr,
                "weight_decay": muon_weight_decay if muon_weight_decay is not None else weight_decay,
                "momentum": muon_momentum, "nesterov": muon_nesterov, "ns_steps": ns_steps, "split": split,
                "update_scale": update_scale}]
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay, use_muon=False)
        super().__init__(all_groups, defaults)
        self.fused_adamw = fused_adamw
        self.ns_dtype = getattr(torch, ns_dtype)
        self._plan = None
        self.exchange = None  # optional replacement of the bf16 all-gather of Muon updates (ddp mode)
        # zero mode (nano_gpic_b200.parallel.ddp): ids of the parameters this rank owns; the step touches only those,
        # Muon orthogonalises all their units locally (their reduced gradients are whole on this rank)
        self.owned = None
        # fused apply (zero mode over peer memory): for the parameters in `defer["ids"]` the step leaves the Muon
        # output O in the flat bf16 buffer defer["upd"] and keeps AdamW state as views of defer["m1"] / defer["m2"];
        # the data-parallel layer's kernel applies both (and the weight broadcast). `deferred` holds this step's
        # scalars for it.
        self.defer = None
        self.deferred = None
        # an attached EMA (train.ema.SimpleEMA.attach): the update kernels also move the EMA of every parameter they
        # update, so no separate pass over the weights is needed
        self.ema = None
        self.applies_ema = True
        self._adam_t = {}  # AdamW step count per group index, on the host (bias corrections of the table kernel)

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        self._adam_t = {}  # re-read from the loaded step tensors

    def _ema_of(self, p):
        return self.ema.view(p) if self.ema is not None else None

    @staticmethod
    def update_coef(group, shape):
        rows, cols = shape
        if group.get("update_scale", "moonlight") == "mup":
            return math.sqrt(rows / cols)
        return 0.2 * math.sqrt(max(rows, cols))

    def _build_plan(self, group):
        """Units (matrix parts), their owner ranks (longest processing time first, cost rows*cols*min) and offsets in
        each owner's flat slot. Deterministic on every rank."""
        world = dist.get_world_size() if dist.is_initialized() else 1
        units = []
        for i, p in enumerate(group["params"]):
            parts = p._muon_parts if group["split"] else 1
            rows = p.shape[0] // parts
            for k in range(parts):
                units.append({"p": i, "r0": k * rows, "r1": (k + 1) * rows, "shape": (rows, p.shape[1])})
        load = [0.0] * world
        order = sorted(range(len(units)), key=lambda j: (-math.prod(units[j]["shape"]) * min(units[j]["shape"]), j))
        for j in order:
            r = min(range(world), key=lambda q: (load[q], q))
            units[j]["owner"] = r
            load[r] += math.prod(units[j]["shape"]) * min(units[j]["shape"])
        offsets = [0] * world
        for u in units:
            u["off"] = offsets[u["owner"]]
            offsets[u["owner"]] += math.prod(u["shape"])
        shard = max(offsets) if offsets else 0
        rank = dist.get_rank() if dist.is_initialized() else 0
        mine = {}
        for u in units:
            if u["owner"] == rank:
                mine.setdefault(u["shape"], []).append(u)
        return {"world": world, "rank": rank, "units": units, "shard": shard, "mine": mine}

    @torch.no_grad()
    def _muon_step_owned(self, group):
        params = [p for p in group["params"] if id(p) in self.owned]
        if not params:
            return
        grads, bufs = [], []
        for p in params:
            st = self.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            grads.append(p.grad)
            bufs.append(st["momentum_buffer"])
        beta, lr, wd = group["momentum"], group["lr"], group["weight_decay"]
        by_shape = {}
        for i, p in enumerate(params):
            parts = p._muon_parts if group["split"] else 1
            rows = p.shape[0] // parts
            for k in range(parts):
                by_shape.setdefault((rows, p.shape[1]), []).append((i, k * rows, (k + 1) * rows))
        outs = []
        # the units cover every row of every owned matrix once: the momentum update happens in the gather's pass,
        # which writes the Newton-Schulz input straight in its precision
        for shape, us in by_shape.items():
            ins = OPT.stack_nesterov([grads[i][r0:r1] for i, r0, r1 in us], [bufs[i][r0:r1] for i, r0, r1 in us],
                                     beta, group["nesterov"], update_momentum=True, dtype=self.ns_dtype)
            O = msign(ins, steps=group["ns_steps"], dtype=self.ns_dtype)
            outs.append((shape, us, O.contiguous() if O.is_cuda else O))
        if self.defer is not None:  # the fused kernel applies W <- W (1 - lr wd) - lr coef O
            d = self.defer
            for shape, us, O in outs:
                for (i, r0, r1), o in zip(us, O):
                    p = params[i]
                    base = d["off"][id(p)] + r0 * p.shape[1]
                    d["upd"][base:base + o.numel()].copy_(o.reshape(-1))
            self.deferred = dict(self.deferred or {}, lr_m=lr, wd_m=wd or 0.0)
            return
        # weight decay and W += coef O for every unit in one launch (units partition each matrix's rows)
        items = [(params[i][r0:r1], o, -lr * self.update_coef(group, shape),
                  None if self.ema is None else self._ema_of(params[i])[r0:r1])
                 for shape, us, O in outs for (i, r0, r1), o in zip(us, O)]
        OPT.apply_updates(items, 1 - lr * wd if wd else 1.0, self.ema.weight if self.ema is not None else 0.0)

    @torch.no_grad()
    def _muon_step(self, group):
        if self.owned is not None:
            return self._muon_step_owned(group)
        params = group["params"]
        grads, bufs = [], []
        for p in params:
            g = p.grad if p.grad is not None else torch.zeros_like(p)
            st = self.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            grads.append(g)
            bufs.append(st["momentum_buffer"])
        beta, lr, wd = group["momentum"], group["lr"], group["weight_decay"]
        if self._plan is None:
            self._plan = self._build_plan(group)
        plan = self._plan
        dev = params[0].device
        single = plan["world"] == 1
        if not single:  # every rank keeps every momentum buffer; with one rank the gather's pass updates them
            torch._foreach_lerp_(bufs, grads, 1 - beta)
        shard = None if single else torch.zeros(plan["shard"], dtype=self.ns_dtype, device=dev)
        local = {}  # one rank: each unit's update straight from the Newton-Schulz output
        for shape, us in plan["mine"].items():
            ins = OPT.stack_nesterov([grads[u["p"]][u["r0"]:u["r1"]] for u in us],
                                     [bufs[u["p"]][u["r0"]:u["r1"]] for u in us], beta, group["nesterov"],
                                     update_momentum=single, dtype=self.ns_dtype)
            O = msign(ins, steps=group["ns_steps"], dtype=self.ns_dtype)
            O = O.contiguous() if O.is_cuda else O
            for u, o in zip(us, O):
                if single:
                    local[(u["p"], u["r0"])] = o
                else:
                    shard[u["off"]:u["off"] + o.numel()].copy_(o.reshape(-1))
        if not single:
            full = self.exchange(shard, plan) if self.exchange is not None else self._all_gather(shard, plan)
        items = []
        for u in plan["units"]:
            if single:
                src = local[(u["p"], u["r0"])]
            else:
                o0 = u["owner"] * plan["shard"] + u["off"]
                src = full[o0:o0 + math.prod(u["shape"])].view(u["shape"])
            ema = None if self.ema is None else self._ema_of(params[u["p"]])[u["r0"]:u["r1"]]
            items.append((params[u["p"]][u["r0"]:u["r1"]], src, -lr * self.update_coef(group, u["shape"]), ema))
        # weight decay and W += coef O for every unit in one launch (units partition each matrix's rows)
        OPT.apply_updates(items, 1 - lr * wd if wd else 1.0, self.ema.weight if self.ema is not None else 0.0)

    @staticmethod
    def _all_gather(shard, plan):
        full = torch.empty(plan["world"] * plan["shard"], dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(full, shard)
        return full

    @torch.no_grad()
    def _adamw_deferred(self, group):
        """AdamW state of the fused-apply parameters as views of the flat buffers; the step count and this step's
        scalars for the kernel."""
        d = self.defer
        steps = []
        for p in group["params"]:
            if id(p) not in d["ids"]:
                continue
            st = self.state[p]
            if "exp_avg" not in st:
                o = d["off"][id(p)]
                st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                st["exp_avg"] = d["m1"][o:o + p.numel()].view(p.shape)
                st["exp_avg_sq"] = d["m2"][o:o + p.numel()].view(p.shape)
            steps.append(st["step"])
        if steps:
            torch._foreach_add_(steps, 1.0)
        d["steps"] = d.get("steps", 0) + 1
        b1, b2 = group["betas"]
        t = d["steps"]
        self.deferred = dict(self.deferred or {}, lr_a=group["lr"], wd_a=group["weight_decay"], b1=b1, b2=b2,
                             eps=group["eps"], bc1=1 - b1 ** t, rsqrt_bc2=(1 - b2 ** t) ** -0.5)

    @torch.no_grad()
    def _adamw_step(self, group):
        from torch.optim.adam import adam as _adam_fn
        if self.defer is not None:
            self._adamw_deferred(group)
        params, grads, m1, m2, steps = [], [], [], [], []
        for p in group["params"]:
            if p.grad is None or (self.owned is not None and id(p) not in self.owned):
                continue
            if self.defer is not None and id(p) in self.defer["ids"]:
                continue
            st = self.state[p]
            if not st:
                st["step"] = (torch.zeros((), dtype=torch.float32, device=p.device) if self.fused_adamw
                              else torch.tensor(0.0, dtype=torch.float32))
                st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            if self.fused_adamw and st["step"].device != p.device:
                st["step"] = st["step"].to(p.device, torch.float32)
            params.append(p)
            grads.append(p.grad)
            m1.append(st["exp_avg"])
            m2.append(st["exp_avg_sq"])
            steps.append(st["step"])
        if not params:
            return
        b1, b2 = group["betas"]
        fused = self.fused_adamw and params[0].is_cuda
        if fused or self.ema is not None:
            # one launch for every parameter of the group (csrc/optim.cu adamw_apply), with the attached EMA; the
            # step tensors stay current for checkpoints, the bias corrections come from a host-side count
            torch._foreach_add_(steps, 1.0)
            gi = next(i for i, g in enumerate(self.param_groups) if g is group)
            t = self._adam_t[gi] + 1 if gi in self._adam_t else int(float(steps[0]))
            self._adam_t[gi] = t
            OPT.adamw_update(params, grads, m1, m2, [self._ema_of(p) for p in params], group["lr"],
                             group["weight_decay"], b1, b2, group["eps"], 1 - b1 ** t, 1 - b2 ** t,
                             self.ema.weight if self.ema is not None else 0.0)
            return
        _adam_fn(params, grads, m1, m2, [], steps, foreach=None if fused else True, capturable=False,
                 differentiable=False, fused=fused or None, grad_scale=None, found_inf=None, has_complex=False,
                 decoupled_weight_decay=True, amsgrad=False, beta1=b1, beta2=b2, lr=group["lr"],
                 weight_decay=group["weight_decay"], eps=group["eps"], maximize=False)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            if group.get("use_muon"):
                self._muon_step(group)
            else:
                self._adamw_step(group)
        return loss
