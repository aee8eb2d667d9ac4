"""Shared helpers for the GPU layer tests: oracle weights from an ExpertBank."""
import numpy as np
import torch

from oracle import moe as OM
from oracle import quant as OQ


def oracle_expert_fn(bank):
    """e -> fp32 (w13, w2) dequantised on the CPU from the bank's packed tiers."""
    cache = {}

    def fn(e):
        if e in cache:
            return cache[e]
        tier, a, b = bank.expert_reference_format(e)
        if tier == "INT4":
            wa = OQ.dequant_int4(a[0].cpu().numpy(), a[1].cpu().numpy())
            wb = OQ.dequant_int4(b[0].cpu().numpy(), b[1].cpu().numpy())
        elif tier == "INT8":
            wa = OQ.dequant_int8(a[0].cpu().numpy(), a[1].cpu().numpy())
            wb = OQ.dequant_int8(b[0].cpu().numpy(), b[1].cpu().numpy())
        else:
            wa = a.float().cpu().numpy()
            wb = b.float().cpu().numpy()
        out = (torch.from_numpy(np.asarray(wa, np.float32)), torch.from_numpy(np.asarray(wb, np.float32)))
        if len(cache) < 16:
            cache[e] = out
        return out
    return fn


def extended_routing(topk_ids, topk_weights, n_routed, n_shared):
    """Append the always-on shared experts as extra top-k columns of weight 1."""
    if n_shared == 0:
        return topk_ids, topk_weights
    t = topk_ids.shape[0]
    sid = torch.arange(n_routed, n_routed + n_shared, dtype=topk_ids.dtype).expand(t, n_shared)
    sw = torch.ones(t, n_shared, dtype=topk_weights.dtype)
    return torch.cat([topk_ids, sid], 1), torch.cat([topk_weights, sw], 1)


def oracle_layer(bank, hidden, topk_ids, topk_weights, tokens=None):
    """fp32 oracle output of the bank's layer (optionally on a token subset)."""
    hid = hidden.cpu()
    ids = topk_ids.cpu().long()
    w = topk_weights.cpu().float()
    if tokens is not None:
        hid, ids, w = hid[tokens], ids[tokens], w[tokens]
    ids, w = extended_routing(ids, w, bank.n_routed, bank.n_shared)
    return OM.moe_layer(hid, ids, w, oracle_expert_fn(bank), None, act_dtype=bank.act_dtype)
