"""Sample rebalancing over ranks by caption length (the roles of the reference's levers E and E2:
baselines/PixelGen/src/utils/rebalance.py:1-142 and src/data/rebalance_loader.py:1-312; both off in its ladder).

Each rank pads its micro-batch's captions to its longest one, and a data-parallel step waits for the slowest rank, so a
rank that drew long captions slows every rank. Here the ranks exchange the samples of a micro-batch so that every rank
keeps the same number of samples and about the same number of caption tokens:

* plan: every rank learns all ranks' caption lengths (one small all_gather of host integers over gloo: no device
  sync), then runs the same deterministic deal: samples in decreasing length order, each to the rank with the fewest
  caption tokens so far among the ranks that still have room. A sample may move to any rank: t and noise are drawn
  per rank, and the gradient is the same sum over the same samples either way (up to fp32 summation order).
* exchange: one all_to_all of the images (uint8, as the loader delivers them: 196 KB per 256 px image instead of the
  reference's 786 KB fp32) and one of the caption rows, padded to the longest caption over all ranks; each rank then
  trims to its own new longest caption and rebuilds the left-aligned mask from the lengths.

Device tensors go through the default process group (NCCL), host tensors through a gloo group (the E2 form: the
exchange runs on the host before the copy to the device, so the GPU never waits for it).
"""
import torch
import torch.distributed as dist


def deal(all_lens, B):
    """all_lens[r][i]: caption length of sample i of rank r (every rank has B). Returns dst[r][i], the rank that
    sample (r, i) goes to; every rank receives exactly B samples."""
    world = len(all_lens)
    order = sorted(((all_lens[r][i], r, i) for r in range(world) for i in range(B)), key=lambda t: (-t[0], t[1], t[2]))
    load, count = [0] * world, [0] * world
    dst = [[0] * B for _ in range(world)]
    for n, r, i in order:
        d = min((k for k in range(world) if count[k] < B), key=lambda k: (load[k], k))
        dst[r][i] = d
        load[d] += n
        count[d] += 1
    return dst


class Rebalancer:
    """rebalance(images, captions, mask) -> (images, captions, mask) after the exchange; a no-op on one rank.
    images [B, ...] (any dtype), captions [B, T, D], mask [B, T] bool left-aligned; all on one device or all on the
    host. `pad_multiple`: the new caption length is rounded up to a multiple of it (the loader's padding rule)."""

    def __init__(self, pad_multiple=8):
        self.pad_multiple = pad_multiple
        self.gloo = None
        self.last_loads = None  # (before, after): per-rank caption tokens of the last call, for logging

    def _group(self, host):
        if not host:
            return None
        if self.gloo is None:
            self.gloo = dist.new_group(backend="gloo")
        return self.gloo

    def __call__(self, images, captions, mask):
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
            return images, captions, mask
        world, me = dist.get_world_size(), dist.get_rank()
        B, T, D = captions.shape
        host = images.device.type == "cpu"
        lens = mask.sum(1).cpu()  # a device mask costs one sync; the loader's host mask does not
        objs = [None] * world
        dist.all_gather_object(objs, [int(x) for x in lens.tolist()], group=self._group(True))
        dst = deal(objs, B)
        loads_after = [0] * world
        for r in range(world):
            for i in range(B):
                loads_after[dst[r][i]] += objs[r][i]
        self.last_loads = ([sum(o) for o in objs], loads_after)
        Tmax = max(max(o) for o in objs)
        Tmax = max(self.pad_multiple, -(-Tmax // self.pad_multiple) * self.pad_multiple)
        # send buffers grouped by destination; received in source-rank order, each source's samples in position order
        send = sorted(range(B), key=lambda i: (dst[me][i], i))
        send_counts = [sum(1 for i in range(B) if dst[me][i] == d) for d in range(world)]
        recv_from = [(r, i) for r in range(world) for i in range(B) if dst[r][i] == me]
        recv_counts = [sum(1 for r, _ in recv_from if r == s) for s in range(world)]
        idx = torch.tensor(send, device=images.device)
        group = self._group(host)
        img_out = torch.empty_like(images)
        dist.all_to_all_single(img_out, images.index_select(0, idx).contiguous(),
                               [c for c in recv_counts], [c for c in send_counts], group=group)
        cap = torch.zeros(B, Tmax, D, dtype=captions.dtype, device=captions.device)
        cap[:, :min(T, Tmax)] = captions[:, :Tmax]
        if host and cap.dtype not in (torch.float32, torch.uint8):
            cap = cap.view(torch.uint8)  # gloo has no 16-bit types: the rows travel as their bytes
        cap_out = torch.empty_like(cap)
        dist.all_to_all_single(cap_out, cap.index_select(0, idx).contiguous(), recv_counts, send_counts, group=group)
        cap_out = cap_out.view(captions.dtype)
        new_lens = torch.tensor([objs[r][i] for r, i in recv_from])
        Tn = max(self.pad_multiple, -(-int(new_lens.max()) // self.pad_multiple) * self.pad_multiple)
        Tn = min(Tn, Tmax)
        new_mask = (torch.arange(Tn)[None, :] < new_lens[:, None]).to(mask.device)
        return img_out, cap_out[:, :Tn].contiguous(), new_mask


PACK_BUCKET = 128


def pack_captions(captions, mask, lens=None, bucket=PACK_BUCKET):
    """Packed captions in the reference's y_pack format (baselines/PixelGen/src/utils/rebalance.py:39-44 and
    JiT_T2I.py:54-65): the real caption tokens of the batch back to back, their count rounded up to a multiple of
    `bucket` with zero dummy rows (so the caption GEMMs see few distinct row counts).

    captions [B, T, D], mask [B, T] bool left-aligned; lens: the host list of caption lengths when the caller has it
    (else one read of the mask). Returns (y [S, D], y_pack) with y_pack = {lens [B] int32, cu [B + 1] int32, pidx [S]
    int64 (b * T + pos; B * T for a dummy row), kmask [B, T] bool, onehot [S, B] bool, real [S] bool, pos [S] int64,
    max_T}, all on the captions' device."""
    B, T, D = captions.shape
    dev = captions.device
    if lens is None:
        lens = [int(v) for v in mask.sum(1).tolist()]
    s_real = sum(lens)
    S = max(bucket, -(-s_real // bucket) * bucket)
    rows = torch.cat([torch.arange(n, dtype=torch.int64) + b * T for b, n in enumerate(lens)] +
                     [torch.full((S - s_real,), B * T, dtype=torch.int64)])
    owner = torch.cat([torch.full((n,), b, dtype=torch.int64) for b, n in enumerate(lens)] +
                      [torch.full((S - s_real,), -1, dtype=torch.int64)])
    real = torch.arange(S) < s_real
    pos = torch.where(real, rows % T, torch.zeros_like(rows))
    onehot = torch.zeros(S, B, dtype=torch.bool)
    onehot[torch.arange(s_real), owner[:s_real]] = True
    lens_t = torch.tensor(lens, dtype=torch.int32)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens_t, 0)
    flat = captions.reshape(B * T, D)
    y = torch.zeros(S, D, dtype=captions.dtype, device=dev)
    y[:s_real] = flat.index_select(0, rows[:s_real].to(dev))
    y_pack = {"lens": lens_t.to(dev), "cu": cu.to(dev), "pidx": rows.to(dev),
              "kmask": (torch.arange(T)[None] < lens_t[:, None]).to(dev), "onehot": onehot.to(dev),
              "real": real.to(dev), "pos": pos.to(dev), "max_T": T}
    return y, y_pack
