"""Reference-compatible hook: the algorithm and payload of the reference's
``python/nangila_ddp/comm_hook.py`` restated with torch ops.

Kept identical on purpose (a payload written by either side must decode the
same way with the other's decoder):

* global absmax scale ``max/qmax`` with qmax 7 (INT4) or 127 (INT8)
  (comm_hook.py:21-25, :177);
* stochastic rounding ``floor(x + U - 0.5)`` with ``U`` from a
  ``torch.Generator`` seeded ``seed ^ (bucket << 16) ^ (call << 32)`` (momentum)
  or ``seed ^ (call << 32)``; the call counter advances once per hook call
  (comm_hook.py:192-205);
* INT4 nibbles, element 2i high (:83-93); top-k byte mask, bit i of byte j =
  element 8j+i (:106-114); values packed in ``torch.topk(sorted=False)`` order
  and decoded in ascending mask order (:180-188, :276-280);
* static topology keep-set from ``randperm`` seeded ``topo_seed ^ (bucket<<16)``
  (:149-174);
* average = prediction + sum of dequantized residuals / world, EMA update
  with the average (:290-299).

Differences: one ``all_gather`` of a fixed-size ``[scale | mask | values]``
record instead of five (every rank's sizes are equal for a bucket), and no
``.item()`` host syncs except for the optional ``res_mean_abs`` metric.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def absmax_scale(x: torch.Tensor, qmax: int) -> torch.Tensor:
    m = torch.nan_to_num(x.abs().max(), nan=0.0, posinf=0.0, neginf=0.0) if x.numel() else torch.zeros((), device=x.device)
    return torch.where(m > 1e-9, m / float(qmax), torch.ones_like(m))


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    if q.numel() % 2:
        q = torch.cat([q, q.new_zeros(1)])
    q = q.view(-1, 2)
    return (((q[:, 0] & 0x0F).to(torch.uint8) << 4) | (q[:, 1] & 0x0F).to(torch.uint8)).contiguous()


def unpack_int4(packed: torch.Tensor, length: int) -> torch.Tensor:
    hi = ((packed >> 4) & 0x0F).to(torch.int8)
    lo = (packed & 0x0F).to(torch.int8)
    hi = (hi << 4) >> 4
    lo = (lo << 4) >> 4
    out = torch.stack([hi, lo], dim=1).reshape(-1)
    return out[:length]


def pack_mask(mask: torch.Tensor) -> torch.Tensor:
    pad = (-mask.numel()) % 8
    if pad:
        mask = torch.cat([mask, mask.new_zeros(pad)])
    m = mask.view(-1, 8).to(torch.uint8)
    weights = (1 << torch.arange(8, device=m.device, dtype=torch.int32)).to(torch.uint8)
    return (m * weights).sum(dim=1, dtype=torch.int32).to(torch.uint8).contiguous()


def unpack_mask(packed: torch.Tensor, length: int) -> torch.Tensor:
    if packed.numel() == 0:
        return torch.zeros(length, dtype=torch.bool, device=packed.device)
    bits = torch.stack([(packed >> i) & 1 for i in range(8)], dim=1).reshape(-1)
    return bits[:length].to(torch.bool)


def topology_keep_mask(nn: int, drop: float, topo_seed: int, bidx: int, device) -> torch.Tensor:
    keep = max(1, int(nn * (1.0 - drop)))
    g = torch.Generator(device=device)
    g.manual_seed((topo_seed ^ (bidx << 16)) & 0xFFFFFFFFFFFFFFFF)
    perm = torch.arange(nn, device=device)[torch.randperm(nn, generator=g, device=device)]
    m = torch.zeros(nn, dtype=torch.bool, device=device)
    m[perm[:keep]] = True
    return m


class CompatCodec:
    """Encoder/decoder of the reference hook's per-bucket payload."""

    def __init__(self, bits=4, stochastic=True, seed=12345, use_momentum=False, topk_percent=0.0,
                 topo_drop_percent=0.0, topo_seed=424242):
        self.bits, self.stochastic, self.seed = bits, stochastic, seed
        self.use_momentum, self.topk_percent = use_momentum, topk_percent
        self.topo_drop_percent, self.topo_seed = topo_drop_percent, topo_seed
        self.call = 0
        self.topo_masks: dict[int, torch.Tensor] = {}

    @property
    def qmax(self) -> int:
        return 7 if self.bits == 4 else 127

    def topo(self, bidx: int, nn: int, device) -> torch.Tensor | None:
        if self.topo_drop_percent <= 0.0:
            return None
        t = self.topo_masks.get(bidx)
        if t is None or t.numel() != nn:
            t = topology_keep_mask(nn, self.topo_drop_percent, self.topo_seed, bidx, device)
            self.topo_masks[bidx] = t
        return t

    def encode(self, residual: torch.Tensor, bidx: int):
        """Returns (scale f32 scalar tensor, packed mask u8, packed values u8)."""
        dev = residual.device
        topo = self.topo(bidx, residual.numel(), dev)
        r = residual[topo] if topo is not None else residual
        qmax = self.qmax
        if self.topk_percent > 0.0:
            n_base = r.numel()
            k = max(1, int(n_base * self.topk_percent))
            _, top_idx = torch.topk(r.abs(), k, sorted=False)
            mask = torch.zeros(n_base, dtype=torch.uint8, device=dev)
            mask[top_idx] = 1
            kept = r[top_idx]
            scale = absmax_scale(kept, qmax)
            scaled = kept / scale
        else:
            mask = None
            scale = absmax_scale(r, qmax)
            scaled = r / scale
        if self.stochastic:
            self.call += 1
            if self.use_momentum:
                seed_mix = self.seed ^ (bidx << 16) ^ (self.call << 32)
            else:
                seed_mix = self.seed ^ (self.call << 32)
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed_mix & 0xFFFFFFFFFFFFFFFF)
            noise = torch.rand(scaled.shape, device=dev, generator=gen, dtype=scaled.dtype) - 0.5
            q = torch.clamp((scaled + noise).floor(), min=-qmax - 1, max=qmax).to(torch.int8)
        else:
            q = torch.clamp(torch.round(scaled), min=-qmax - 1, max=qmax).to(torch.int8)
        vals = pack_int4(q) if self.bits == 4 else q.view(torch.uint8)
        pm = pack_mask(mask.bool()) if mask is not None else torch.empty(0, dtype=torch.uint8, device=dev)
        return scale.float().reshape(()), pm, vals

    def decode(self, scale: torch.Tensor, pm: torch.Tensor, pv: torch.Tensor, nn: int, bidx: int) -> torch.Tensor:
        """Dequantized residual of one rank (fp32, length nn)."""
        dev = pv.device
        topo = self.topo(bidx, nn, dev)
        if pm.numel() > 0:
            base_len = nn if topo is None else int(topo.sum())
            mask_r = unpack_mask(pm, base_len)
            kc = int(mask_r.sum())
            qi = unpack_int4(pv, kc).float() if self.bits == 4 else pv.view(torch.int8).float()[:kc]
            res = torch.zeros(nn, dtype=torch.float32, device=dev)
            if topo is not None:
                rt = res[topo]
                rt[mask_r] = qi * scale
                res[topo] = rt
            else:
                res[mask_r] = qi * scale
            return res
        qi = unpack_int4(pv, nn).float() if self.bits == 4 else pv.view(torch.int8).float()[:nn]
        if topo is not None:
            res = torch.zeros(nn, dtype=torch.float32, device=dev)
            res[topo] = qi[: int(topo.sum())] * scale
            return res
        return qi * scale


def make_compat_hook(hs):
    cfg = hs.config
    codec = CompatCodec(cfg.bits, cfg.stochastic, cfg.seed, cfg.use_momentum, cfg.topk_percent,
                        cfg.topo_drop_percent, cfg.topo_seed)
    states: dict[int, torch.Tensor] = {}
    hs.codec = codec
    hs.compat_states = states

    @torch.no_grad()
    def hook(_state, bucket):
        from .hook import _log

        buf = bucket.buffer()
        bidx = bucket.index()
        world = dist.get_world_size(hs.group)
        prev = states.get(bidx) if cfg.use_momentum else None
        if prev is not None and prev.shape == buf.shape:
            pred = prev
        else:
            pred = torch.zeros_like(buf)
        residual = buf - pred
        scale, pm, pv = codec.encode(residual, bidx)
        record = torch.cat([scale.reshape(1).view(torch.uint8), pm, pv])
        gathered = [torch.empty_like(record) for _ in range(world)]
        dist.all_gather(gathered, record, group=hs.group)
        nm = pm.numel()
        res_sum = torch.zeros(buf.numel(), dtype=torch.float32, device=buf.device)
        for r in range(world):
            rec = gathered[r]
            s = rec[:4].view(torch.float32)[0]
            res_sum.add_(codec.decode(s, rec[4:4 + nm], rec[4 + nm:], buf.numel(), bidx))
        reduced = (pred.to(torch.float32) + res_sum / float(world)).to(buf.dtype)
        if cfg.use_momentum:
            if prev is not None and prev.shape == reduced.shape:
                prev.mul_(cfg.beta).add_(reduced, alpha=1.0 - cfg.beta)
            else:
                states[bidx] = reduced.clone()
        hs.calls += 1
        comp = pv.numel() + nm + 4
        hs.raw_bytes += buf.numel() * 4
        hs.comp_bytes += comp
        if cfg.metrics_path or cfg.verbose:
            _log(hs, bidx, buf.numel(), comp, float(residual.abs().mean()))
        fut = torch.futures.Future()
        fut.set_result(reduced)
        return fut

    return hook
