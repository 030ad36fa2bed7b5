"""Exponential moving average of the weights (reference baselines/PixelGen/src/callbacks/simple_ema.py:12-111).

ema <- decay * ema + (1 - decay) * w once per optimizer step, as one lerp over the flat fp32 parameter buffer on a side
stream, joined before the next optimizer step and before any checkpoint. With off=True (the ladder: GPIC_MFU_NO_EMA=1)
nothing is updated and checkpoints mirror the raw weights into the EMA slot.
"""
import os

import torch


class SimpleEMA:
    def __init__(self, flat, decay=0.9999, every_n_steps=1, off=None, ranges=None):
        self.flat = flat
        # zero mode: only these [start, end) ranges of the flat buffer are current on this rank (its owned segments
        # and the replicated bucket), so only they are averaged; a checkpoint gathers the rest from their owners
        self.ranges = ranges
        self.decay, self.every_n_steps = decay, every_n_steps
        self.off = (os.environ.get("GPIC_MFU_NO_EMA") == "1") if off is None else off
        self.buf = None if self.off else flat.data.clone()
        self._stream = None
        self.previous_step = 0
        self.fused = False  # True once attach() handed the update to the optimizer's kernels
        self._index = None

    @property
    def weight(self):
        return 1.0 - self.decay

    def view(self, p):
        """The EMA tensor of parameter p (a view of the flat EMA buffer)."""
        if self._index is None:
            self._index = {id(q): i for i, q in enumerate(self.flat.params)}
        return self.flat.view(self.buf, self._index[id(p)])

    def attach(self, opt):
        """Let the optimizer's update kernels apply the EMA in the same pass as the weight update (the role of the
        reference's FusedAdamWEMA with an EMA, baselines/PixelGen/src/utils/fused_adamw_ema.py:39-113): the same
        lerp, one pass over the weights fewer. Only for an EMA updated every step; returns whether it attached."""
        if self.off or self.every_n_steps != 1 or not self.buf.is_cuda or not getattr(opt, "applies_ema", False):
            return False
        opt.ema = self
        self.fused = True
        return True

    def step(self, global_step):
        """Call after the optimizer step; updates once per new step (nothing to do when attached to the optimizer,
        whose kernels updated it)."""
        if self.off or global_step == self.previous_step:
            return
        self.previous_step = global_step
        if self.fused:
            return
        if global_step % self.every_n_steps:
            return
        if self.buf.is_cuda:
            if self._stream is None:
                self._stream = torch.cuda.Stream(device=self.buf.device)
            self._stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._stream):
                self._lerp()
        else:
            self._lerp()

    def _lerp(self):
        if self.ranges is None:
            self.buf.lerp_(self.flat.data, 1.0 - self.decay)
            return
        for a, b in self.ranges:
            self.buf[a:b].lerp_(self.flat.data[a:b], 1.0 - self.decay)

    def join(self):
        if self._stream is not None:
            torch.cuda.current_stream().wait_stream(self._stream)

    def state_tensors(self, prefix):
        """The EMA weights under the denoiser's parameter names (non-trainable buffers/params as the model has them)."""
        self.join()
        model = self.flat.module
        out = {}
        ema_of = {id(p): self.flat.view(self.buf, i) for i, p in enumerate(self.flat.params)}
        for k, v in model.state_dict(keep_vars=True).items():
            out[prefix + k] = ema_of.get(id(v), v).detach()
        return out

    def load_tensors(self, sd):
        if self.off:
            return
        names = dict(zip(self.flat.names, range(len(self.flat.params))))
        for k, v in sd.items():
            if k in names:
                self.flat.view(self.buf, names[k]).copy_(v)

    def state_dict(self):
        return {"decay": self.decay, "every_n_steps": self.every_n_steps}

    def load_state_dict(self, sd):
        self.decay, self.every_n_steps = sd["decay"], sd["every_n_steps"]
