"""Caption conditioners: they turn captions (or the batch's cached encoder outputs) into the denoiser's caption
features [B, T, embed_dim] bf16 and the padding mask, and give the null caption for guidance.

    BaseConditioner           __call__(y, metadata) -> (condition, uncondition), floats cast to bf16
                              (reference baselines/PixelGen/src/models/conditioner/base.py)
    ComposeConditioner        concatenation of several along T
    CachedTextConditioner     the training path: the batch already carries the frozen encoder's outputs
                              (metadata text_emb / text_mask, read from the text cache by the data loader), so no
                              encoder runs in the step (reference src/models/conditioner/cached_text.py)
    Qwen3TextEncoder          the online encoder for prediction and for building the cache: a transformers Qwen3Model
                              (last hidden state), right padding to the longest caption rounded up to pad_multiple,
                              features cut or zero-padded to embed_dim; the null caption is one EOS token
                              (reference src/models/conditioner/qwen3_text_encoder.py, text_mode "masked")
"""
import os

import torch

from ..data.text_cache import assert_left_aligned


class BaseConditioner(torch.nn.Module):
    def _impl_condition(self, y, metadata):
        raise NotImplementedError

    def _impl_uncondition(self, y, metadata):
        raise NotImplementedError

    @torch.no_grad()
    def __call__(self, y, metadata=None):
        metadata = {} if metadata is None else metadata
        cond = self._impl_condition(y, metadata)
        uncond = self._impl_uncondition(y, metadata)
        if cond.dtype in (torch.float64, torch.float32, torch.float16):
            cond = cond.to(torch.bfloat16)
        if uncond.dtype in (torch.float64, torch.float32, torch.float16):
            uncond = uncond.to(torch.bfloat16)
        return cond, uncond


class ComposeConditioner(BaseConditioner):
    def __init__(self, conditioners):
        super().__init__()
        self.conditioners = conditioners

    def _impl_condition(self, y, metadata):
        return torch.cat([c._impl_condition(y, metadata) for c in self.conditioners], dim=1)

    def _impl_uncondition(self, y, metadata):
        return torch.cat([c._impl_uncondition(y, metadata) for c in self.conditioners], dim=1)


def _to_device(t, device):
    if device is None or t.device == torch.device(device):
        return t
    if t.device.type == "cpu" and torch.device(device).type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


class CachedTextConditioner(BaseConditioner):
    """Reads metadata["text_emb"] [B, T, D] bf16 and metadata["text_mask"] [B, T]; sets metadata["y_mask"]. The null
    caption is emb_dir/null.pt ([1, 1, D] bf16: the encoder's output for one EOS token) at position 0, zeros after."""

    def __init__(self, emb_dir=None, embed_dim=2048, device=None):
        super().__init__()
        self.embed_dim, self.device = embed_dim, device
        path = os.path.join(emb_dir, "null.pt") if emb_dir else None
        if path and os.path.exists(path):
            self.null_cpu = torch.load(path, map_location="cpu", weights_only=True)
            assert self.null_cpu.dtype == torch.bfloat16 and self.null_cpu.shape == (1, 1, embed_dim)
        else:
            self.null_cpu = torch.zeros(1, 1, embed_dim, dtype=torch.bfloat16)
        self._null = {}

    def _impl_condition(self, y, metadata):
        dev = self.device or metadata["text_emb"].device
        out = _to_device(metadata["text_emb"], dev)
        mask = _to_device(metadata["text_mask"], dev).bool()
        metadata["y_mask"] = mask
        assert_left_aligned(mask)
        return out

    def _impl_uncondition(self, y, metadata):
        dev = metadata["y_mask"].device
        if dev not in self._null:
            self._null[dev] = self.null_cpu.to(dev)
        T = metadata["y_mask"].shape[1]
        out = torch.zeros(len(y), T, self.embed_dim, device=dev, dtype=torch.bfloat16)
        out[:, 0] = self._null[dev][0, 0]
        return out


class Qwen3TextEncoder(BaseConditioner):
    """weight_path: a local Hugging Face Qwen3 directory (tokenizer + model). `model`/`tokenizer` may be given
    directly (e.g. a randomly initialised Qwen3Model from a config, and any callable tokenizer)."""

    def __init__(self, weight_path=None, embed_dim=None, max_length=128, pad_multiple=8, model=None, tokenizer=None,
                 device=None):
        super().__init__()
        if model is None or tokenizer is None:
            from transformers import AutoTokenizer, Qwen3Model
            tokenizer = tokenizer or AutoTokenizer.from_pretrained(weight_path, padding_side="right")
            model = model or Qwen3Model.from_pretrained(weight_path, torch_dtype=torch.bfloat16)
        self.tokenizer, self.model = tokenizer, model.to(torch.bfloat16).eval()
        if device is not None:
            self.model.to(device)
        self.embed_dim = embed_dim or self.model.config.hidden_size
        self.max_length, self.pad_multiple = max_length, pad_multiple
        self.null_embedding = None

    @property
    def _dev(self):
        return next(self.model.parameters()).device

    def _fit_dim(self, y):
        D = y.shape[2]
        if D < self.embed_dim:
            y = torch.cat([y, y.new_zeros(y.shape[0], y.shape[1], self.embed_dim - D)], dim=-1)
        return y[:, :, :self.embed_dim]

    def tokenize(self, captions):
        tok = self.tokenizer(list(captions), truncation=True, max_length=self.max_length, padding="longest",
                             pad_to_multiple_of=self.pad_multiple, return_tensors="pt")
        return tok["input_ids"], tok["attention_mask"].bool()

    @torch.no_grad()
    def encode(self, input_ids, mask):
        dev = self._dev
        input_ids, mask = _to_device(input_ids, dev), _to_device(mask, dev)
        out = self.model(input_ids=input_ids, attention_mask=mask.long())[0]
        return self._fit_dim(out.to(torch.bfloat16)), mask

    def _impl_condition(self, y, metadata):
        if metadata.get("input_ids") is not None:  # tokenized in the data workers
            ids, mask = metadata["input_ids"], metadata["text_mask"].bool()
        else:
            ids, mask = self.tokenize(y)
        out, mask = self.encode(ids, mask)
        metadata["y_mask"] = mask
        assert_left_aligned(mask)
        return out

    def null(self):
        """The encoder's output for one EOS token, [1, 1, embed_dim] bf16 (the cache's null.pt)."""
        if self.null_embedding is None:
            eos = getattr(self.tokenizer, "eos_token_id", None)
            eos = 0 if eos is None else eos
            ids = torch.tensor([[eos]])
            self.null_embedding, _ = self.encode(ids, torch.ones_like(ids, dtype=torch.bool))
        return self.null_embedding

    def _impl_uncondition(self, y, metadata):
        nul = self.null()
        T = metadata["y_mask"].shape[1] if "y_mask" in metadata else 1
        out = torch.zeros(len(y), T, self.embed_dim, device=nul.device, dtype=nul.dtype)
        out[:, 0] = nul[0, 0]
        return out
