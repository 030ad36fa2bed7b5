"""Flat parameter storage: every trainable parameter of a module becomes a view of one fp32 buffer, its gradient a view
of one fp32 gradient buffer, and its bf16 compute copy a view of one bf16 buffer.

Why: the kernels accumulate weight gradients straight into `.grad` (no autograd accumulation pass), the data-parallel
layer reduces contiguous buckets of the gradient buffer without copies, the optimizer kernels walk one buffer, and
refreshing the bf16 compute weights after a step is one cast kernel. The parameters keep their identity and names, so
state dicts, optimizer state and checkpoints are unchanged (the reference's DDP `gradient_as_bucket_view=True` plays
the same role for its gradients; baselines/PixelGen/configs_h100/lite_ladder.yaml:7-12).

Every view starts on a multiple of ALIGN elements (16-byte alignment of the bf16 views for TMA).
"""
import torch

ALIGN = 64


def _round(n, a=ALIGN):
    return (n + a - 1) // a * a


class FlatParams:
    """params/offsets/numel: an explicit layout (e.g. the data-parallel planner's bucket and owner order, with padding);
    by default the module's trainable parameters back to back."""

    def __init__(self, module, device=None, params=None, offsets=None, numel=None, grad_buf=None, data16_buf=None):
        self.module = module
        self.params = list(params) if params is not None else [p for p in module.parameters() if p.requires_grad]
        names = {id(p): n for n, p in module.named_parameters()}
        self.names = [names.get(id(p), f"param{i}") for i, p in enumerate(self.params)]
        device = device or self.params[0].device
        if offsets is None:
            self.offsets = []
            off = 0
            for p in self.params:
                self.offsets.append(off)
                off = _round(off + p.numel())
        else:
            assert len(offsets) == len(self.params) and all(o % ALIGN == 0 for o in offsets)
            self.offsets = list(offsets)
            off = numel
            assert all(o + p.numel() <= off for o, p in zip(self.offsets, self.params))
        self.numel = off
        self.data = torch.zeros(off, dtype=torch.float32, device=device)
        # grad_buf / data16_buf: externally allocated storage (e.g. peer-shared memory), zero-filled, >= numel elements
        self.grad = grad_buf[:off] if grad_buf is not None else torch.zeros(off, dtype=torch.float32, device=device)
        self.data16 = (data16_buf[:off] if data16_buf is not None
                       else torch.zeros(off, dtype=torch.bfloat16, device=device))
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.data[o:o + n].copy_(p.detach().reshape(-1).to(device=device, dtype=torch.float32))
            p.data = self.data[o:o + n].view(p.shape)
            p.grad = self.grad[o:o + n].view(p.shape)
            p._bf16 = self.data16[o:o + n].view(p.shape)
        self.sync_bf16()

    def view(self, buf, i):
        p, o = self.params[i], self.offsets[i]
        return buf[o:o + p.numel()].view(p.shape)

    def sync_bf16(self):
        """Refresh the bf16 compute weights from the fp32 master weights (after an optimizer step or a load)."""
        self.data16.copy_(self.data)

    def zero_grad(self):
        self.grad.zero_()

    def grad_norm(self):
        return self.grad.norm()

    def ranges(self, bucket_numel):
        """Contiguous [start, end) ranges of the flat buffers, about bucket_numel elements each, on parameter
        boundaries, in reverse parameter order (the order the backward produces gradients)."""
        out, end = [], self.numel
        start = end
        for o in reversed(self.offsets):
            start = o
            if end - start >= bucket_numel:
                out.append((start, end))
                end = start
        if end > 0:
            out.append((0, end))
        return out
