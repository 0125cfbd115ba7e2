"""Partition of the token-mixer work across the GPUs of one node.

Both kernels are sums of independent units, so the GPUs share no data on the hot path:
  * flash_attention_2: a (batch, key/value head) unit with the query heads of its group;
  * qwen35moe_gdn_prefill: a (sequence, value head) unit; value head h reads key head h % Hk, so a
    group of key heads together with every value head that reads them is self-contained.
Each rank runs the unmodified kernel on its slice.  The only communication is the gather of the
outputs (and final states) to rank 0 for verification, outside any timed region.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def even_ranges(n: int, world: int) -> list[tuple[int, int]]:
    """Split range(n) into `world` contiguous [a, b) ranges whose sizes differ by at most one."""
    if world <= 0:
        raise ValueError("world must be positive")
    base, extra = divmod(n, world)
    out, a = [], 0
    for r in range(world):
        b = a + base + (1 if r < extra else 0)
        out.append((a, b))
        a = b
    return out


def gdn_value_heads(a: int, b: int, hk: int, hv: int) -> list[int]:
    """Value heads that read key heads [a, b) (h % hk in [a, b)), ordered so that local value
    head i reads local key head i % (b - a) -- the kernel's own head mapping on the slice."""
    if hv % hk != 0:
        raise ValueError("hv must be a multiple of hk")
    return [h for rep in range(hv // hk) for h in range(rep * hk + a, rep * hk + b)]


def slice_gdn_inputs(inp: dict, a: int, b: int) -> dict:
    """Inputs of the GDN plugin restricted to key heads [a, b) and the value heads reading them."""
    hk, hv = inp["q"].shape[2], inp["v"].shape[2]
    vh = gdn_value_heads(a, b, hk, hv)
    out = dict(inp)
    out["q"] = inp["q"][:, :, a:b].contiguous()
    out["k"] = inp["k"][:, :, a:b].contiguous()
    idx = torch.tensor(vh, device=inp["v"].device)
    for key in ("v", "g", "beta"):
        out[key] = inp[key].index_select(2, idx).contiguous()
    if inp.get("state") is not None:
        out["state"] = inp["state"].index_select(1, idx.to(inp["state"].device)).contiguous()
    return out


def slice_fa2_inputs(inp: dict, a: int, b: int) -> dict:
    """FA2 plugin inputs restricted to key/value heads [a, b) and their query heads."""
    layout = inp.get("layout", "bhsd")
    hd = 1 if layout == "bhsd" else 2
    group = inp["q"].shape[hd] // inp["k"].shape[hd]
    out = dict(inp)
    out["q"] = inp["q"].narrow(hd, a * group, (b - a) * group).contiguous()
    out["k"] = inp["k"].narrow(hd, a, b - a).contiguous()
    out["v"] = inp["v"].narrow(hd, a, b - a).contiguous()
    return out


def gather_to_rank0(local: torch.Tensor, dim: int):
    """All-gather per-rank slices (possibly of different sizes along `dim`) and concatenate them
    on rank 0 in rank order; other ranks get None.  Verification only (never timed)."""
    if not (dist.is_available() and dist.is_initialized()):
        return local
    world = dist.get_world_size()
    sizes = [None] * world
    dist.all_gather_object(sizes, int(local.shape[dim]))
    pad = max(sizes) - local.shape[dim]
    if pad:
        shape = list(local.shape)
        shape[dim] = pad
        local = torch.cat([local, local.new_zeros(shape)], dim=dim)
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous())
    if dist.get_rank() != 0:
        return None
    return torch.cat([p.narrow(dim, 0, n) for p, n in zip(parts, sizes)], dim=dim)


def unscatter_gdn_heads(parts: list[torch.Tensor], ranges: list[tuple[int, int]], hk: int, hv: int,
                        dim: int) -> torch.Tensor:
    """Put the value-head slices of every rank back in global head order along `dim`."""
    order = [h for a, b in ranges for h in gdn_value_heads(a, b, hk, hv)]
    cat = torch.cat(parts, dim=dim)
    inv = torch.empty(len(order), dtype=torch.long)
    inv[torch.tensor(order)] = torch.arange(len(order))
    return cat.index_select(dim, inv.to(cat.device))
