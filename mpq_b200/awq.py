"""AWQ activation-aware scaling, the preprocess of the 3/4-bit recipe (mpq/awq_scale.py:49-816).

Per decoder layer and projection group (q/k/v after the attention norm, o after v, gate/up after the MLP norm,
down after up) a per-input-channel scale s is searched over 20 ratios r = 0, 0.05, ..., 0.95:
s = clamp(x_mean^r / (w_mean^(1-r) + 1e-4), 1e-4) / sqrt(max(s) min(s)), where x_mean is the mean |x| of the
group's calibration inputs and w_mean the mean group-normalised |W| (times the previous group's mean |W| for
the o, gate/up and down groups); the group's weights are scaled, pseudo-quantized on the asymmetric (or
symmetric) group grid and unscaled, the inspected module is run on the captured inputs, and the ratio with the
smallest mean squared output error wins (first minimum).  The scales are then folded into the preceding norm or
linear (norm weight / s, linear rows / s) and the group's weights (columns * s), which leaves the float model's
function unchanged.  Calibration activations stay on the GPU; the module forwards are the model's own.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence

import torch


def _pseudo_quantize_(w: torch.Tensor, bits: int, group_size: int, sym: bool) -> None:
    """In place, in w's dtype (mpq/awq_scale.py:109-157)."""
    v = w.view(-1, group_size) if group_size > 0 else w.view(w.shape[0], -1)
    if not sym:
        mx = v.amax(dim=1, keepdim=True)
        mn = v.amin(dim=1, keepdim=True)
        max_int = 2 ** bits - 1
        s = (mx - mn).clamp(min=1e-5) / max_int
        z = (-torch.round(mn / s)).clamp_(0, max_int)
        v.div_(s)
        torch.round(v, out=v)
        v.add_(z).clamp_(0, max_int).sub_(z).mul_(s)
    else:
        mx = v.abs().amax(dim=1, keepdim=True).clamp(min=1e-5)
        max_int = 2 ** (bits - 1) - 1
        s = mx / max_int
        v.div_(s)
        torch.round(v, out=v)
        v.clamp_(-(2 ** (bits - 1)), max_int).mul_(s)


def _w_mean(linears: Sequence[torch.nn.Linear], group_size: int) -> torch.Tensor:
    """mpq/awq_scale.py:49-82: mean over rows of |W| normalised by its group maximum (+1e-6)."""
    w0 = linears[0].weight
    acc = torch.zeros(w0.shape[1], dtype=torch.float32, device=w0.device)
    rows = 0
    for fc in linears:
        w = fc.weight
        if group_size > 0:
            if w.shape[-1] % group_size:
                raise ValueError(f"weight shape {tuple(w.shape)} is not divisible by group_size={group_size}")
            g = w.abs().view(-1, group_size)
        else:
            g = w.abs().reshape(w.shape[0], -1)
        norm = (g / (g.amax(dim=1, keepdim=True) + 1e-6)).view(w.shape)
        acc += norm.sum(dim=0, dtype=torch.float32)
        rows += w.shape[0]
    return (acc / max(rows, 1)).to(w0.dtype)


def _candidate(x_mean: torch.Tensor, w_mean: torch.Tensor, ratio: float) -> torch.Tensor:
    """mpq/awq_scale.py:338-347."""
    s = (x_mean.pow(ratio) / (w_mean.pow(1 - ratio) + 1e-4)).clamp(min=1e-4)
    s = s / (s.max() * s.min()).sqrt()
    s[torch.isinf(s)] = 1
    s[torch.isnan(s)] = 1
    return s


def _search(linears: Sequence[torch.nn.Linear], x: torch.Tensor, run, group_size: int, bits: int, sym: bool,
            hint: Optional[float]):
    """mpq/awq_scale.py:491-580: the best of 20 ratios for one group; returns (scales, error, ratio)."""
    flat = x.abs().reshape(-1, x.shape[-1]).to(torch.float32)
    x_mean = (flat.sum(dim=0) / max(int(flat.shape[0]), 1)).to(x.dtype)
    w_mean = _w_mean(linears, group_size)
    if hint is not None:
        w_mean = w_mean * float(hint)
    orig = [fc.weight.detach().clone() for fc in linears]
    fp = run(x)
    fp = fp.clip(torch.finfo(fp.dtype).min, torch.finfo(fp.dtype).max)
    best, best_err, best_ratio = None, float("inf"), -1.0
    for ri in range(20):
        ratio = ri / 20.0
        s = _candidate(x_mean, w_mean, ratio)
        sv = s.view(1, -1)
        for fc in linears:
            fc.weight.mul_(sv.to(fc.weight.dtype))
            _pseudo_quantize_(fc.weight.data, bits, group_size, sym)
            fc.weight.div_(sv.to(fc.weight.dtype))
        out = run(x)
        out = out.clip(torch.finfo(out.dtype).min, torch.finfo(out.dtype).max)
        d = (fp - out).float()
        err = float(d.pow(2).sum().item()) / max(int(d.numel()), 1)
        for fc, w in zip(linears, orig):
            fc.weight.copy_(w)
        if err < best_err:
            best_err, best_ratio, best = err, ratio, s.detach().clone()
    if best is None:
        raise RuntimeError("AWQ scale search failed to find a valid ratio")
    return best, best_err, best_ratio


def _scale_ln_fcs(ln, fcs, s):
    s = s.to(ln.weight.dtype)
    ln.weight.div_(s)
    if getattr(ln, "bias", None) is not None:
        ln.bias.div_(s)
    for fc in fcs:
        fc.weight.mul_(s.view(1, -1).to(fc.weight.dtype))


def _scale_fc_fc(fc1, fc2, s):
    s = s.to(fc1.weight.dtype)
    fc1.weight[-s.size(0):].div_(s.view(-1, 1))
    if fc1.bias is not None:
        fc1.bias.div_(s.view(-1))
    fc2.weight.mul_(s.view(1, -1).to(fc2.weight.dtype))


def _mean_abs(mods) -> float:
    vals = [float(m.weight.detach().abs().mean().item()) for m in mods]
    return float(sum(vals) / max(len(vals), 1))


@torch.no_grad()
def apply_awq_scaling(model, calib_ids: torch.Tensor, *, bits: int, group_size: int = 128, sym: bool = False,
                      batch_size: int = 1) -> Dict[str, Any]:
    """Apply AWQ scaling to a decoder LM in place (mpq/awq_scale.py:591-813).  ``calib_ids`` (samples x seq) are
    the calibration token ids; ``batch_size`` sequences go through each module forward at a time.
    Returns the per-layer search record (best ratio and error per group)."""
    dev = next(model.parameters()).device
    if dev.type != "cuda":
        raise ValueError("apply_awq_scaling runs on the GPU (move the model to a CUDA device)")
    inner = model.model
    n_seq, seq_len = calib_ids.shape
    bs = max(int(batch_size), 1)
    hidden = inner.embed_tokens(calib_ids.to(dev))
    pos_ids = torch.arange(seq_len, device=dev)[None]
    pos_emb = inner.rotary_emb(hidden[:1], position_ids=pos_ids)

    def batched(fn, x):
        return torch.cat([fn(x[b0:b0 + bs]) for b0 in range(0, x.shape[0], bs)], dim=0)

    layers_dbg: List[Dict[str, Any]] = []
    for li, layer in enumerate(inner.layers):
        def attn(x, _sa=layer.self_attn):
            return _first(_sa(hidden_states=x, position_embeddings=pos_emb, attention_mask=None))

        sa, mlp = layer.self_attn, layer.mlp
        q, k, v, o = sa.q_proj, sa.k_proj, sa.v_proj, sa.o_proj
        gate, up, down = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        cap: Dict[str, List[torch.Tensor]] = {"qkv_x": [], "o_x": [], "gate_x": [], "down_x": []}
        hooks = [q.register_forward_pre_hook(lambda m, a: cap["qkv_x"].append(a[0].detach())),
                 o.register_forward_pre_hook(lambda m, a: cap["o_x"].append(a[0].detach())),
                 gate.register_forward_pre_hook(lambda m, a: cap["gate_x"].append(a[0].detach())),
                 down.register_forward_pre_hook(lambda m, a: cap["down_x"].append(a[0].detach()))]
        try:
            for b0 in range(0, n_seq, bs):
                layer(hidden[b0:b0 + bs], attention_mask=None, position_embeddings=pos_emb, position_ids=pos_ids)
        finally:
            for h in hooks:
                h.remove()
        xs = {k_: torch.cat(v_, dim=0) for k_, v_ in cap.items()}
        qkv_hint = _mean_abs([q, k, v])
        o_hint = _mean_abs([o])
        gu_hint = _mean_abs([gate, up])
        same_vo = v.weight.shape == o.weight.shape
        pending, groups = [], []
        s, err, ratio = _search([q, k, v], xs["qkv_x"], lambda x: batched(attn, x), group_size, bits, sym, None)
        pending.append(("qkv", s))
        groups.append({"name": "qkv", "prev_op": "input_layernorm", "best_ratio": ratio, "best_error": err})
        if same_vo:
            s, err, ratio = _search([o], xs["o_x"], lambda x: batched(o, x), group_size, bits, sym, qkv_hint)
            pending.append(("o_proj", s))
            groups.append({"name": "o_proj", "prev_op": "v_proj", "best_ratio": ratio, "best_error": err})
        s, err, ratio = _search([gate, up], xs["gate_x"], lambda x: batched(mlp, x), group_size, bits, sym,
                                o_hint if same_vo else None)
        pending.append(("gate_up", s))
        groups.append({"name": "gate_up", "prev_op": "post_attention_layernorm", "best_ratio": ratio,
                       "best_error": err})
        s, err, ratio = _search([down], xs["down_x"], lambda x: batched(down, x), group_size, bits, sym, gu_hint)
        pending.append(("down_proj", s))
        groups.append({"name": "down_proj", "prev_op": "up_proj", "best_ratio": ratio, "best_error": err})
        del xs, cap
        for name, s in pending:
            if name == "qkv":
                _scale_ln_fcs(layer.input_layernorm, [q, k, v], s)
            elif name == "o_proj":
                _scale_fc_fc(v, o, s)
            elif name == "gate_up":
                _scale_ln_fcs(layer.post_attention_layernorm, [gate, up], s)
            else:
                _scale_fc_fc(up, down, s)
        nxt = torch.empty_like(hidden)
        for b0 in range(0, n_seq, bs):
            nxt[b0:b0 + bs] = _first(layer(hidden[b0:b0 + bs], attention_mask=None, position_embeddings=pos_emb,
                                           position_ids=pos_ids))
        hidden = nxt
        layers_dbg.append({"layer_index": li, "groups": groups})
    return {"layers": layers_dbg, "bits": int(bits), "group_size": int(group_size), "sym": bool(sym),
            "batch_size": bs}


def _first(out):
    return out[0] if isinstance(out, (tuple, list)) else out
