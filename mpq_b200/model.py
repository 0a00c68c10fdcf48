"""Whole-model quantization driver for decoder LMs (GPTQModel-style sequential layer walk).

The reference reaches a whole model through GPTQModel's processor loop, which collects each linear's
Hessian with forward hooks (GPTQ.add_batch) and calls MPQ's ``run_mpq_quantization`` per linear
(patches/gptqmodel.patch:672-756, mpq/adapters/gptqmodel.py:650-1163), and through the QUIP# driver for
E8P12 (mpq/quip_generic.py).  This module restates that walk on the B200 kernels:

* layers are processed in order; inside a layer the linears are quantized in GPTQ's sequential subsets
  ([q, k, v], [o], [gate, up], [down]) and each subset's Hessian is collected with the already-quantized
  subsets in place (``true_sequential``), then the layer's outputs with quantized weights feed the next layer;
* Hessian hooks feed bfloat16 activations straight into the tensor-core X^T X (exact TF32 operands); linears
  fed by the same input share one Hessian and one eigendecomposition;
* with N ranks (one process per GPU) the calibration sequences are split across ranks, the partial sums
  X^T X and sample counts are all-reduced (NCCL over NVLink), every linear's output rows are solved as row
  shards, and the dequantized rows are all-gathered so every rank holds the quantized layer.

The model shapes of the synthetic benchmark configs are in ``CONFIGS`` (random init, std 0.02).
"""
from __future__ import annotations

import time
import types
from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import ops
from .hessian import accumulate_xtx
from .pipeline import SetupPipeline
from .shard import gather_rows, row_shards

CONFIGS: Dict[str, Dict[str, Any]] = {
    # Qwen3-0.6B shape
    "qwen3_0p6b": dict(family="qwen3", hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, vocab_size=151936),
    # Llama-3.2-1B shape
    "llama32_1b": dict(family="llama", hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, vocab_size=128256),
    # Llama-3-8B shape
    "llama3_8b": dict(family="llama", hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, vocab_size=128256),
    # small shape for tests
    "tiny_llama": dict(family="llama", hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64, vocab_size=1000),
}

SUBSETS = (("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), ("self_attn.o_proj",),
           ("mlp.gate_proj", "mlp.up_proj"), ("mlp.down_proj",))


def build_synthetic_decoder(name: str, *, device, seed: int = 0, num_layers: Optional[int] = None,
                            dtype=torch.bfloat16):
    """Random-init (std 0.02) decoder LM of a registered shape, built directly on `device`."""
    from transformers import AutoModelForCausalLM, LlamaConfig, Qwen3Config
    spec = dict(CONFIGS[name])
    fam = spec.pop("family")
    if num_layers is not None:
        spec["num_hidden_layers"] = int(num_layers)
    cls = Qwen3Config if fam == "qwen3" else LlamaConfig
    cfg = cls(initializer_range=0.02, attn_implementation="sdpa", max_position_embeddings=4096, **spec)
    torch.manual_seed(int(seed))
    with torch.device(device):
        model = AutoModelForCausalLM.from_config(cfg, dtype=dtype)
    return model.eval()


def calibration_ids(n_seq: int, seq_len: int, vocab: int, seed: int = 0) -> torch.Tensor:
    """Uniform-random token ids (n_seq x seq_len), the synthetic calibration set."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randint(0, int(vocab), (int(n_seq), int(seq_len)), generator=g)


@dataclass
class ModelQuantConfig:
    bits: int = 4
    group_size: int = 128
    rotation_mode: str = "internal_hadamard"
    iters: int = 20
    prior_tau: float = 0.2
    damping: float = 0.5
    polish_sweeps: int = 3
    polish_mode: str = "block_cd"  # "block_cd" | "topk_block_cd" | "none"
    topk_k: int = 16
    init: str = "rtn"  # "rtn" | "float" (VAMP's starting message)
    block_cd_backend: str = "auto"
    true_sequential: bool = True
    batch_size: int = 8          # calibration sequences per forward
    keep_codes: bool = False     # gather q_int / scale / zero of every linear to the host
    export_gptq: bool = False    # also pack them into GPTQ v1 tensors (qweight / qzeros / scales / g_idx)
    checkpoint_dir: Optional[str] = None  # per-layer resume state: layer_<i>.pt after each layer; done layers load
    keep_inputs: bool = False    # keep every linear's solve inputs (float W, its Hessian) on the host (checking)


def _world(group=None) -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


class _Timer:
    def __init__(self, dev):
        self.dev, self.acc = dev, {}

    def __call__(self, name):
        timer = self

        class _Ctx:
            def __enter__(self):
                torch.cuda.synchronize(timer.dev)
                self.t = time.perf_counter()

            def __exit__(self, *a):
                torch.cuda.synchronize(timer.dev)
                timer.acc[name] = timer.acc.get(name, 0.0) + time.perf_counter() - self.t
        return _Ctx()


class _StopForward(Exception):
    """Raised by the last Hessian hook of a subset: the rest of the layer's forward is not needed."""


def _forward_layer(layer, hidden, out, bs, mask, pos_emb, pos_ids):
    for b0 in range(0, hidden.shape[0], bs):
        o = layer(hidden[b0:b0 + bs], attention_mask=mask, position_embeddings=pos_emb, position_ids=pos_ids)
        if out is not None:
            out[b0:b0 + bs].copy_(o)


@torch.inference_mode()
def quantize_model(model, calib_ids: torch.Tensor, cfg: ModelQuantConfig, *, group=None,
                   layers: Optional[Sequence[int]] = None) -> Dict[str, Any]:
    """Quantize every linear of every decoder layer in place (weights replaced by their dequantized values).

    Returns {"modules": {name: stats (+ codes when keep_codes)}, "timings": {...}, "seconds": wall}."""
    from .adapters.gptqmodel import GPTQAdapterConfig, run_mpq_quantization
    from .solver import UniformVampConfig
    rank, world = _world(group)
    dev = next(model.parameters()).device
    timer = _Timer(dev)
    t_start = time.perf_counter()
    inner = model.model
    n_seq, seq_len = calib_ids.shape
    s0, s1 = row_shards(n_seq, world, 1)[rank]
    ids = calib_ids[s0:s1].to(dev)
    qcfg = types.SimpleNamespace(bits=int(cfg.bits), group_size=int(cfg.group_size), desc_act=False,
                                 mpq=types.SimpleNamespace(rotation_mode=cfg.rotation_mode, solver="vamp"))
    vcfg = UniformVampConfig(iters=int(cfg.iters), prior_tau=float(cfg.prior_tau), damping=float(cfg.damping),
                             polish_sweeps=int(cfg.polish_sweeps), polish_mode=str(cfg.polish_mode),
                             topk_k=int(cfg.topk_k), init_from=str(cfg.init), block_cd_backend=cfg.block_cd_backend)
    with timer("embed"):
        hidden = inner.embed_tokens(ids)
        nxt = torch.empty_like(hidden)
    pos_ids = torch.arange(seq_len, device=dev)[None]
    pos_emb = inner.rotary_emb(hidden[:1], position_ids=pos_ids)
    mask = None  # sdpa causal attention without padding
    results: Dict[str, Any] = {}
    layer_ids = list(range(len(inner.layers))) if layers is None else list(layers)
    for li in layer_ids:
        layer = inner.layers[li]
        if _resume_layer(cfg.checkpoint_dir, li, layer, results, rank, world, group):
            with timer("forward_out"):
                _forward_layer(layer, hidden, nxt, int(cfg.batch_size), mask, pos_emb, pos_ids)
            hidden, nxt = nxt, hidden
            continue
        subsets = SUBSETS if cfg.true_sequential else (sum(SUBSETS, ()),)
        for subset in subsets:
            # keyed by the Hessian's address: valid only while this subset's Hessians are alive
            eigen_cache: dict = {}
            mods = {name: layer.get_submodule(name) for name in subset}
            # the linears of a subset read the same input (q/k/v: the attention norm's output, gate/up: the MLP
            # norm's output): one Hessian per distinct input, collected on its first reader
            readers: Dict[int, str] = {}
            for name, m in mods.items():
                readers.setdefault(id(_input_owner(layer, name)), name)
            sums: Dict[str, torch.Tensor] = {}
            counts: Dict[str, int] = {}

            last_reader = list(readers.values())[-1]

            def make_hook(name):
                def hook(mod, args):
                    x = args[0]
                    S = sums.get(name)
                    if S is None:
                        S = sums[name] = torch.zeros(x.shape[-1], x.shape[-1], device=dev, dtype=torch.float32)
                        counts[name] = 0
                    accumulate_xtx(S, x, alpha=1.0, beta=1.0)
                    counts[name] += int(x.shape[0]) if x.dim() == 3 else 1  # GPTQ counts leading-dim samples
                    if name == last_reader:
                        raise _StopForward()
                return hook

            handles = [mods[name].register_forward_pre_hook(make_hook(name)) for name in readers.values()]
            with timer("forward_hessian"):
                for b0 in range(0, hidden.shape[0], int(cfg.batch_size)):
                    try:
                        layer(hidden[b0:b0 + int(cfg.batch_size)], attention_mask=mask, position_embeddings=pos_emb,
                              position_ids=pos_ids)
                    except _StopForward:
                        pass
            for h in handles:
                h.remove()
            Hs: Dict[str, torch.Tensor] = {}
            with timer("hessian_reduce"):
                for name, S in sums.items():  # GPTQ convention H = 2 / nsamples * sum x x^T, over all ranks
                    cnt = torch.tensor([float(counts[name])], device=dev, dtype=torch.float64)
                    if world > 1:
                        dist.all_reduce(S, group=group)
                        dist.all_reduce(cnt, group=group)
                    S.mul_(2.0 / float(cnt.item()))
                for name in mods:
                    Hs[name] = sums[readers[id(_input_owner(layer, name))]]
            for name, m in mods.items():
                full = f"model.layers.{li}.{name}"
                W = m.weight
                rows = W.shape[0]
                r0, r1 = row_shards(rows, world, 128)[rank]
                with timer("solve"):
                    if r1 > r0:
                        Wl = W[r0:r1].to(torch.float32)
                        acfg = GPTQAdapterConfig(block_rows=r1 - r0, grow_block_rows=False, eigen_cache=eigen_cache)
                        Q, q_int, scale, zero, g_idx, secs, st = run_mpq_quantization(
                            W=Wl, H=Hs[name], quantizer=None, qcfg=qcfg, module_name=full, vamp_cfg=vcfg,
                            adapter_cfg=acfg)
                    else:  # more ranks than row tiles: nothing to solve here
                        ng = (W.shape[1] + int(cfg.group_size) - 1) // int(cfg.group_size)
                        Q = torch.empty(0, W.shape[1], device=dev)
                        q_int = torch.empty(0, W.shape[1], device=dev, dtype=torch.uint8)
                        scale = zero = torch.empty(0, ng, device=dev)
                        g_idx = torch.arange(W.shape[1], device=dev, dtype=torch.int32) // int(cfg.group_size)
                        secs, st = 0.0, {}
                with timer("gather"):
                    Qa = gather_rows(Q.to(W.dtype).contiguous(), row_shards(rows, world, 128), group=group)
                    inputs = {"W": W.float().cpu(), "H": Hs[name].float().cpu()} if cfg.keep_inputs else None
                    W.copy_(Qa)
                    lr = max(r1 - r0, 1)
                    entry = {"rows": rows, "cols": W.shape[1], "rows_local": (r0, r1), "solve_s": secs,
                             "rankspace_error_mean": st.get("stabilized_objective_mean_final"),
                             "rtn_rankspace_error_mean": st.get("rtn_error_sum", 0.0) / lr,
                             "raw_objective_mean": st.get("raw_objective_mean_final")}
                    if cfg.keep_codes or cfg.export_gptq:
                        sh = row_shards(rows, world, 128)
                        qa = gather_rows(q_int, sh, group=group)
                        sa = gather_rows(scale.contiguous(), sh, group=group)
                        za = gather_rows(zero.contiguous(), sh, group=group)
                        if cfg.keep_codes:
                            entry.update(q_int=qa.cpu(), scale=sa.cpu(), zero=za.cpu(), g_idx=g_idx.cpu())
                        if cfg.export_gptq:
                            from .export import pack_gptq
                            entry["gptq"] = {k: v.cpu() for k, v in pack_gptq(qa, sa, za, g_idx, int(cfg.bits)).items()}
                    if inputs is not None:
                        entry["inputs"] = inputs
                    results[full] = entry
            del sums, Hs
        if cfg.checkpoint_dir and rank == 0:
            _save_layer(cfg.checkpoint_dir, li, layer, {k: v for k, v in results.items()
                                                        if k.startswith(f"model.layers.{li}.")})
        with timer("forward_out"):
            _forward_layer(layer, hidden, nxt, int(cfg.batch_size), mask, pos_emb, pos_ids)
        hidden, nxt = nxt, hidden
    ops.check_status(dev)
    torch.cuda.synchronize(dev)
    return {"modules": results, "timings": dict(timer.acc), "seconds": time.perf_counter() - t_start}


def _layer_path(ckpt_dir: str, li: int) -> str:
    import os
    return os.path.join(ckpt_dir, f"layer_{li}.pt")


def _save_layer(ckpt_dir: str, li: int, layer, entries: Dict[str, Any]) -> None:
    """The resume state of one finished layer: its quantized (dequantized) linear weights and module entries,
    written to a temporary name and renamed so that a partial file is never taken for a finished layer."""
    import os
    os.makedirs(ckpt_dir, exist_ok=True)
    weights = {name: layer.get_submodule(name).weight.detach().cpu() for name in sum(SUBSETS, ())}
    path = _layer_path(ckpt_dir, li)
    torch.save({"weights": weights, "modules": entries}, path + ".tmp")
    os.replace(path + ".tmp", path)


def _resume_layer(ckpt_dir: Optional[str], li: int, layer, results: Dict[str, Any], rank: int, world: int,
                  group) -> bool:
    """Load layer li's saved state when it exists (the decision is rank 0's, shared with every rank)."""
    import os
    if not ckpt_dir:
        return False
    flag = [os.path.isfile(_layer_path(ckpt_dir, li)) if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(flag, src=0, group=group)
    if not flag[0]:
        return False
    state = torch.load(_layer_path(ckpt_dir, li), map_location="cpu", weights_only=False)
    for name, w in state["weights"].items():
        layer.get_submodule(name).weight.copy_(w)
    results.update(state["modules"])
    return True


def _input_owner(layer, name: str):
    """The module whose output is `name`'s input: the attention or MLP pre-norm for the projections that read
    it, otherwise the module itself."""
    if name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
        return layer.input_layernorm
    if name in ("mlp.gate_proj", "mlp.up_proj"):
        return layer.post_attention_layernorm
    return layer.get_submodule(name)


# ------------------------------------------------------------------------------------------------------------------
# QUIP#-style E8P12 walk (mpq/quip_generic.py): Hessians from the float model, fused projection groups,
# randomized Hadamard incoherence on both sides, mpq_refine_codebook per group, checkpoint attribute dicts.
# ------------------------------------------------------------------------------------------------------------------

QUIP_GROUPS = (("qkv", ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")), ("o", ("self_attn.o_proj",)),
               ("up", ("mlp.up_proj", "mlp.gate_proj")), ("down", ("mlp.down_proj",)))


@dataclass
class QuipModelConfig:
    iters: int = 16
    prior_tau: float = 0.25
    damping: float = 0.5
    init: str = "rtn"  # "rtn" | "float"
    polish_sweeps: int = 3
    polish_mode: str = "block_cd"  # "block_cd" | "topk_block_cd" | "none"
    topk_k: int = 16
    sigma_reg: float = 1e-2
    seed: int = 0
    batch_size: int = 8
    write_back: bool = True      # replace the float weights by the dequantized E8P12 weights
    keep_attrs: bool = True      # keep the per-group checkpoint attributes (on the host)
    checkpoint_dir: Optional[str] = None  # QUIP#-layout ckpt: {layer}_{group}.pt / {layer}_layernorm.pt written as
    #                                       layers finish; groups whose file exists are loaded instead of solved
    fingerprint: bool = False    # sha256 of each group's W and H in the ckpt (host hashing: seconds per layer)
    block_rows: int = 128        # the adapter's chained row blocks (mpq/adapters/quip_sharp.py:28)
    keep_inputs: bool = False    # keep every group's solve inputs (rotated unit-RMS W, rotated H) on the host
    pipelined: bool = False      # set up the next group (rotations, eigendecomposition) while a group is solved
    #                              (same results; on B200 the solve keeps the GPU busy, so this measured no faster)


def _quip_group_setup(layer, mods, H, key: str, seed: int, dev) -> Dict[str, Any]:
    """Layer-wide set-up of one projection group: W = vstack(w_i / rms(w_i)), sign vectors seeded by the group's
    name, the two-sided randomized Hadamard of W and H, the unit-RMS scale and the floored fp64 eigendecomposition
    of the rotated Hessian (mpq/quip_generic.py:1012-1046, mpq/adapters/quip_sharp.py:33-67)."""
    from .adapters.gptqmodel import vamp_hessian_eigen
    from .rotation import rht_hessian, rht_weight, sample_rademacher_signs
    ws = [layer.get_submodule(m).weight.to(torch.float32) for m in mods]
    scales = [float(w.square().mean().sqrt().item()) for w in ws]
    W = torch.cat([w / s for w, s in zip(ws, scales)], dim=0).contiguous()
    m, n = W.shape
    SU = sample_rademacher_signs(width=m, key=f"{key}:SU", seed=seed, device=dev)
    SV = sample_rademacher_signs(width=n, key=f"{key}:SV", seed=seed, device=dev)
    Wr = rht_weight(W, SU, SV, m & -m, n & -n)
    Hr = rht_hessian(H, SV, n & -n)
    wscale = float(Wr.square().mean().sqrt().item())
    Wn = (Wr / wscale).contiguous()
    return {"ws": ws, "scales": scales, "W": W, "SU": SU, "SV": SV, "Hr": Hr, "wscale": wscale, "Wn": Wn,
            "eig": vamp_hessian_eigen(Hr, fp64=True)}


@torch.inference_mode()
def quantize_model_quip(model, calib_ids: torch.Tensor, cfg: QuipModelConfig, *, group=None) -> Dict[str, Any]:
    """E8P12 quantization of every decoder layer (2 bits per weight), QUIP#-style.

    Hessians: one float forward per layer with QUIP# hooks (sum x^T x, sum x, token count) on the inputs of
    q (the fused qkv), o, up (the fused up+gate) and down, finalised as H / ct - mu mu^T and re-centred to the
    second moment H / ct (mpq/quip_generic.py:906-918, 373-375), then regularize_H (sigma_reg, :378).  Each group
    W = vstack(w_i / rms(w_i)) gets random sign vectors SU, SV (seeded by the group's name), a two-sided block
    Hadamard, unit RMS scaling and mpq_refine_codebook (RTN init, VAMP, gram-metric CD).  With N ranks the
    calibration sequences are split across ranks (partial sums all-reduced); all layers' Hessians are collected
    first, then layer l's groups are solved on rank l mod N concurrently, the owners broadcast the quantized weights
    and the attributes are gathered on rank 0.  The packed Qidxs layout of QUIP#'s decode kernels is
    QUIP#'s own (not part of the reference tree): Qidxs are kept unpacked (int16, rows x cols / 8)."""
    from .adapters.quip_sharp import mpq_refine_codebook
    from .codebook import E8P12_codebook
    from .hessian import HessianAccumulator, regularize_H
    from .rotation import rht_hessian, rht_weight, rht_weight_inverse, sample_rademacher_signs
    rank, world = _world(group)
    dev = next(model.parameters()).device
    timer = _Timer(dev)
    t_start = time.perf_counter()
    cb = E8P12_codebook()
    inner = model.model
    n_seq, seq_len = calib_ids.shape
    s0, s1 = row_shards(n_seq, world, 1)[rank]
    with timer("embed"):
        hidden = inner.embed_tokens(calib_ids[s0:s1].to(dev))
        nxt = torch.empty_like(hidden)
    pos_ids = torch.arange(seq_len, device=dev)[None]
    pos_emb = inner.rotary_emb(hidden[:1], position_ids=pos_ids)
    args = types.SimpleNamespace(mpq_init=str(cfg.init), mpq_iters=int(cfg.iters), mpq_prior_tau=float(cfg.prior_tau),
                                 mpq_damping=float(cfg.damping),
                                 mpq_polish_sweeps=int(cfg.polish_sweeps), mpq_block_rows=int(cfg.block_rows),
                                 quant_solver="vamp", quant_polish_mode=str(cfg.polish_mode), mpq_polish_metric="gram",
                                 mpq_topk_k=int(cfg.topk_k), seed=int(cfg.seed))
    attrs: Dict[str, Any] = {}
    nl = len(inner.layers)
    done = _quip_done_groups(cfg.checkpoint_dir, nl, rank, world, group)
    # phase 1: every layer's Hessians from the float model (float activations feed the next layer)
    Hs_all: Dict[Tuple[int, str], torch.Tensor] = {}
    for li in range(nl):
        layer = inner.layers[li]
        accs = {name: HessianAccumulator(layer.get_submodule(mods[0]).in_features, device=dev, mode="quip")
                for name, mods in QUIP_GROUPS if f"{li}_{name}" not in done}
        handles = [layer.get_submodule(mods[0]).register_forward_pre_hook(
            (lambda acc: (lambda mod, a: acc.add_batch(a[0])))(accs[name])) for name, mods in QUIP_GROUPS
            if name in accs]
        with timer("forward_hessian"):
            _forward_layer(layer, hidden, nxt, int(cfg.batch_size), None, pos_emb, pos_ids)
        for h in handles:
            h.remove()
        with timer("hessian_reduce"):
            for name, acc in accs.items():
                S, mu = acc.H, acc.mu
                ct = torch.tensor([float(acc.ct)], device=dev, dtype=torch.float64)
                if world > 1:
                    dist.all_reduce(S, group=group)
                    dist.all_reduce(mu, group=group)
                    dist.all_reduce(ct, group=group)
                H = S / float(ct.item())  # = (H / ct - mu mu^T) + mu mu^T with mu = sum x / ct
                Hs_all[(li, name)] = regularize_H(H, H.shape[0], float(cfg.sigma_reg))
            del accs
        hidden, nxt = nxt, hidden
    del hidden, nxt
    # phase 2: layer l is solved on rank l mod N (the layers are independent given the float Hessians); the set-up of
    # the next group runs on the set-up pipeline while a group is solved
    jobs = [(li, name, mods, f"{li}_{name}") for li in range(nl) if li % world == rank for name, mods in QUIP_GROUPS]
    todo = [j for j in jobs if j[3] not in done]
    pipe = SetupPipeline(dev) if (cfg.pipelined and todo) else None

    def queue(j):
        li, name, mods, key = j
        pipe.submit(key, _quip_group_setup, inner.layers[li], mods, Hs_all[(li, name)], key, int(cfg.seed), dev)

    try:
        if pipe is not None:
            queue(todo[0])
        ti = 0
        for li, name, mods, key in jobs:
            layer = inner.layers[li]
            if key in done:
                with timer("resume"):
                    attrs[key] = _quip_load_group(cfg.checkpoint_dir, key, layer, mods, cb, bool(cfg.write_back))
                continue
            with timer("solve"):
                H = Hs_all[(li, name)]
                if pipe is not None:
                    P = pipe.get(key)
                    nxt = todo[ti + 1] if ti + 1 < len(todo) else None
                    after = (lambda j=nxt: queue(j)) if nxt is not None else None
                else:
                    P = _quip_group_setup(layer, mods, H, key, int(cfg.seed), dev)
                    after = None
                ti += 1
                ws, scales, W, SU, SV = P["ws"], P["scales"], P["W"], P["SU"], P["SV"]
                wscale, Wn = P["wscale"], P["Wn"]
                m, n = W.shape
                hat, idx, st = mpq_refine_codebook(Wn, P["Hr"], Wn, torch.zeros(m, n // 8, dtype=torch.int64, device=dev),
                                                   cb, args, module_name=key, eigen=P["eig"], after_enqueue=after)
                hatW = rht_weight_inverse(hat * wscale, SU, SV, m & -m, n & -n)
                if cfg.write_back:
                    r0 = 0
                    for mod_name, w, sc in zip(mods, ws, scales):
                        rows = w.shape[0]
                        layer.get_submodule(mod_name).weight.copy_((hatW[r0:r0 + rows] * sc).to(w.dtype))
                        r0 += rows
                diff = hatW - W
                err_proxy = float(((diff @ H) * diff).sum().item() / max(((W @ H) * W).sum().abs().item(), 1e-12))
                entry = {"fused": len(mods) > 1, "shapes": [tuple(w.shape) for w in ws], "scales": scales,
                         "proxy_error": err_proxy, "surrogate_before": st["exact_surrogate_before_mean"],
                         "surrogate_after": st["exact_surrogate_after_mean"]}
                if cfg.keep_attrs or cfg.checkpoint_dir:
                    entry.update(Qidxs=idx.to(torch.int16).cpu(), SU=SU.to(torch.float16).cpu(),
                                 SV=(SV * wscale).to(torch.float16).cpu(),
                                 mpq_stats={k: v for k, v in st.items() if isinstance(v, (int, float, str, bool))})
                if cfg.fingerprint:
                    from .adapters.gptqmodel import _tensor_sha256
                    entry["input_fingerprint"] = {"protocol": "paired_w_h_sha256_v1", "w_sha256": _tensor_sha256(W),
                                                  "h_sha256": _tensor_sha256(H), "w_shape": [int(d) for d in W.shape],
                                                  "h_shape": [int(d) for d in H.shape], "basis": "pre_incoherence"}
                if cfg.checkpoint_dir:
                    from .export import save_quip_layer
                    save_quip_layer(cfg.checkpoint_dir, li, layer, {name: entry})
                if not cfg.keep_attrs:
                    for k in ("Qidxs", "SU", "SV"):
                        entry.pop(k, None)
                if cfg.keep_inputs:
                    entry["inputs"] = {"Wn": Wn.cpu(), "Hr": P["Hr"].cpu()}
                attrs[key] = entry
                del P
    finally:
        if pipe is not None:
            pipe.close()
    del Hs_all
    # phase 3: every rank holds the quantized model (the owners' weights)
    if world > 1 and cfg.write_back:
        with timer("gather"):
            for li in range(nl):
                layer = inner.layers[li]
                for _, mods in QUIP_GROUPS:
                    for mod_name in mods:
                        dist.broadcast(layer.get_submodule(mod_name).weight, li % world, group=group)
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, {k: {kk: vv for kk, vv in v.items() if not torch.is_tensor(vv)}
                                          for k, v in attrs.items()}, group=group)
        if rank == 0:
            for part in gathered:
                for k, v in part.items():
                    attrs.setdefault(k, v)
    ops.check_status(dev)
    torch.cuda.synchronize(dev)
    return {"groups": attrs, "timings": dict(timer.acc), "seconds": time.perf_counter() - t_start}


def _quip_done_groups(ckpt_dir: Optional[str], nl: int, rank: int, world: int, group) -> set:
    """Groups whose checkpoint file exists (rank 0's view, shared with every rank)."""
    import os
    done = [None]
    if rank == 0:
        done[0] = {f"{li}_{name}" for li in range(nl) for name, _ in QUIP_GROUPS
                   if ckpt_dir and os.path.isfile(os.path.join(ckpt_dir, f"{li}_{name}.pt"))}
    if world > 1:
        dist.broadcast_object_list(done, src=0, group=group)
    return done[0]


def _quip_load_group(ckpt_dir: str, key: str, layer, mods, cb, write_back: bool) -> Dict[str, Any]:
    """Load a finished group and (optionally) write its decoded weights back: W_i = scale_i * rows_i of
    diag(SU) Had^T grid[Qidxs] Had^T diag(SV) (SV carries the RMS scale), the inverse of the incoherence
    processing applied before the solve."""
    import os
    from .codebook import factor_tables
    from .rotation import rht_weight_inverse
    attr = torch.load(os.path.join(ckpt_dir, f"{key}.pt"), map_location="cpu", weights_only=False)
    if write_back:
        dev = layer.get_submodule(mods[0]).weight.device
        # Qidxs are stored as int16 (QUIP#'s dtype): codes >= 2^15 read back negative, so take the low 16 bits
        idx = attr["Qidxs"].to(device=dev, dtype=torch.int64) & 0xFFFF
        m, nb = idx.shape
        n = nb * 8
        grid = factor_tables(cb, dev)["grid"]
        hat = grid.index_select(0, idx.reshape(-1)).reshape(m, n)
        hatW = rht_weight_inverse(hat, attr["SU"].to(dev).float(), attr["SV"].to(dev).float(), m & -m, n & -n)
        r0 = 0
        for mod_name, sc in zip(mods, attr["scales"]):
            w = layer.get_submodule(mod_name).weight
            rows = w.shape[0]
            w.copy_((hatW[r0:r0 + rows] * float(sc)).to(w.dtype))
            r0 += rows
    attr["resumed"] = True
    return attr
