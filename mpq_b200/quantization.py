"""The public entry point: ``QuantizationConfig`` and ``quantize`` (mpq/quantization.py:17-380).

The reference resolves the user configuration to a backend recipe (2 bits: QUIP# E8P12 with randomized
Hadamard; 3/4 bits: GPTQModel grouped scalar with AWQ scaling and the internal Hadamard) and launches the backend
scripts.  Here the same resolution drives the in-process B200 drivers of ``mpq_b200.model``: the model (a loaded
Hugging Face decoder, a local checkpoint directory, or a registered synthetic shape) is calibrated, optionally AWQ-
scaled, quantized layer by layer on the GPU, and written out (GPTQ-format directory or QUIP#-layout ckpt plus the
dense Hugging Face model), with ``backend_results.json`` summarising the run.  Calibration text datasets are not
downloaded: pass ``calibration_ids`` or use ``calibration_dataset="random"`` (uniform token ids).
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Dict, Optional

import torch

SUPPORTED_BITS = (2, 3, 4)
SYNTHETIC_DATASETS = ("random", "synthetic", "uniform")


@dataclass(frozen=True)
class ResolvedQuantizationConfig:
    bits: int
    backend: str
    backend_env: str
    codebook: str
    preprocess: str
    rotation: str
    solver: str
    polish_mode: str
    group_size: int
    symmetric: Optional[bool]
    init: str
    iters: int
    damping: float
    prior_tau: float
    polish_sweeps: int
    calibration_dataset: str
    calibration_samples: int
    calibration_seqlen: int
    seed: int
    evaluate: bool
    save: bool


@dataclass(frozen=True)
class QuantizationConfig:
    """User-facing MPQ configuration; defaults select the paper recipe for each bit width."""

    bits: int = 4
    group_size: int = 128
    preprocess: str = "auto"
    symmetric: Optional[bool] = None
    init: str = "auto"
    iters: int = 16
    damping: float = 0.5
    prior_tau: Optional[float] = None
    polish_sweeps: int = 3
    calibration_dataset: str = "c4"
    calibration_samples: int = 128
    calibration_seqlen: int = 2048
    seed: int = 0
    evaluate: bool = False
    save: bool = True
    backend_env: Optional[str] = None

    def resolve(self) -> ResolvedQuantizationConfig:
        """The backend recipe (mpq/quantization.py:67-150): validation, then bits 2 -> QUIP#/E8P12/"had",
        bits 3 and 4 -> GPTQModel/grid_g128/internal_hadamard (AWQ preprocess unless asked otherwise)."""
        bits = int(self.bits)
        if bits not in SUPPORTED_BITS:
            raise ValueError(f"bits must be one of {SUPPORTED_BITS}; got {bits}")
        if int(self.group_size) <= 0 and int(self.group_size) != -1:
            raise ValueError("group_size must be positive or -1")
        if int(self.calibration_samples) <= 0:
            raise ValueError("calibration_samples must be positive")
        if int(self.calibration_seqlen) <= 0:
            raise ValueError("calibration_seqlen must be positive")
        if int(self.iters) <= 0:
            raise ValueError("iters must be positive")
        if not 0.0 <= float(self.damping) <= 1.0:
            raise ValueError("damping must be in [0, 1]")
        if int(self.polish_sweeps) < 0:
            raise ValueError("polish_sweeps must be non-negative")
        preprocess = str(self.preprocess).strip().lower()
        if preprocess == "auto":
            preprocess = "none" if bits == 2 else "awq"
        if preprocess not in {"none", "awq"}:
            raise ValueError("preprocess must be one of: auto, none, awq")
        init = str(self.init).strip().lower()
        if init == "auto":
            init = "rtn"
        if init not in {"float", "rtn", "random", "ldlq"}:
            raise ValueError("init must be one of: auto, float, rtn, random, ldlq")
        common = dict(bits=bits, solver="vamp", polish_mode="block_cd" if self.polish_sweeps else "none",
                      group_size=int(self.group_size), init=init, iters=int(self.iters), damping=float(self.damping),
                      prior_tau=0.2 if self.prior_tau is None else float(self.prior_tau),
                      polish_sweeps=int(self.polish_sweeps), calibration_dataset=str(self.calibration_dataset),
                      calibration_samples=int(self.calibration_samples),
                      calibration_seqlen=int(self.calibration_seqlen), seed=int(self.seed),
                      evaluate=bool(self.evaluate), save=bool(self.save), preprocess=preprocess)
        if bits == 2:
            return ResolvedQuantizationConfig(
                backend="quip", backend_env=self.backend_env or os.environ.get("MPQ_QUIP_ENV") or "mpq-quip",
                codebook="e8p12", rotation="had", symmetric=None, **common)
        return ResolvedQuantizationConfig(
            backend="gptqmodel", backend_env=self.backend_env or os.environ.get("MPQ_GPTQ_ENV") or "mpq-gptq",
            codebook="grid_g128", rotation="internal_hadamard",
            symmetric=False if self.symmetric is None else bool(self.symmetric), **common)


def _load_model(model, dev, seed: int):
    from .model import CONFIGS, build_synthetic_decoder
    if isinstance(model, torch.nn.Module):
        return model, type(model).__name__
    name = str(model)
    if name in CONFIGS:
        return build_synthetic_decoder(name, device=dev, seed=seed), name
    if os.path.isdir(name):
        from transformers import AutoModelForCausalLM
        m = AutoModelForCausalLM.from_pretrained(name, dtype=torch.bfloat16)
        return m.to(dev).eval(), name
    raise ValueError(f"model {name!r}: pass a loaded model, a local checkpoint directory or one of "
                     f"{sorted(CONFIGS)} (there is no network access for Hugging Face ids)")


def _calibration(resolved: ResolvedQuantizationConfig, vocab: int, calibration_ids) -> torch.Tensor:
    from .model import calibration_ids as synth_ids
    if calibration_ids is not None:
        ids = torch.as_tensor(calibration_ids, dtype=torch.long)
        if ids.dim() != 2:
            raise ValueError("calibration_ids must be (samples, seqlen)")
        return ids
    if resolved.calibration_dataset.strip().lower() in SYNTHETIC_DATASETS:
        return synth_ids(resolved.calibration_samples, resolved.calibration_seqlen, vocab, seed=resolved.seed)
    raise ValueError(f"calibration dataset {resolved.calibration_dataset!r} needs a download: pass calibration_ids "
                     f"or calibration_dataset in {SYNTHETIC_DATASETS}")


def quantize(model, output_dir, config: Optional[QuantizationConfig] = None, *, calibration_ids=None,
             device=None, resume: bool = True, group=None, awq_batch_size: int = 16) -> Dict[str, Any]:
    """Quantize a decoder LM and return the result payload (also written to ``output_dir/backend_results.json``).

    ``model``: a loaded ``*ForCausalLM`` (quantized in place), a local checkpoint directory, or a registered
    synthetic shape name.  With ``resume`` the per-layer state under ``output_dir`` lets an interrupted run skip the
    layers it finished.  Under ``torchrun`` pass the process group in ``group``; rank 0 writes the files.
    ``awq_batch_size`` sequences go through each module forward of the AWQ search (a throughput knob)."""
    import torch.distributed as dist

    from .model import ModelQuantConfig, QuipModelConfig, quantize_model, quantize_model_quip
    t0 = time.time()
    resolved = (config or QuantizationConfig()).resolve()
    if resolved.init in {"random", "ldlq"}:
        raise ValueError(f"init={resolved.init!r} is not on the CUDA path (use 'rtn' or 'float')")
    if resolved.symmetric:
        raise ValueError("symmetric grids are not on the CUDA path (the solve uses the asymmetric GPTQ grid)")
    if resolved.evaluate:
        raise ValueError("evaluate=True runs the reference's text-dataset evaluation scripts, which are not part of "
                         "this package; quantize with evaluate=False and evaluate the saved model separately")
    rank = dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = Path(output_dir).expanduser()
    out.mkdir(parents=True, exist_ok=True)
    m, model_name = _load_model(model, dev, resolved.seed)
    ids = _calibration(resolved, int(m.config.vocab_size), calibration_ids)
    payload: Dict[str, Any] = {"backend": resolved.backend, "model": model_name, "config": asdict(resolved),
                               "calibration": {"samples": int(ids.shape[0]), "seqlen": int(ids.shape[1]),
                                               "dataset": resolved.calibration_dataset if calibration_ids is None
                                               else "user"}}
    timings: Dict[str, float] = {}
    if resolved.preprocess == "awq":
        from .awq import apply_awq_scaling
        t = time.time()
        payload["awq"] = apply_awq_scaling(m, ids, bits=resolved.bits,
                                           group_size=resolved.group_size if resolved.group_size > 0 else -1,
                                           sym=bool(resolved.symmetric), batch_size=awq_batch_size)
        timings["awq_preprocess"] = time.time() - t
    paths: Dict[str, str] = {}
    if resolved.backend == "quip":
        ckpt = out / "quip_ckpt"
        qcfg = QuipModelConfig(iters=resolved.iters, prior_tau=resolved.prior_tau, damping=resolved.damping,
                               init=resolved.init, polish_sweeps=resolved.polish_sweeps, polish_mode=resolved.polish_mode,
                               seed=resolved.seed, keep_attrs=False,
                               checkpoint_dir=str(ckpt) if (resolved.save or resume) else None)
        res = quantize_model_quip(m, ids, qcfg, group=group)
        payload["groups"] = res["groups"]
        if resolved.save and rank == 0:
            from .export import export_dense_hf_from_ckpt, save_quip_config
            save_quip_config(ckpt, m, asdict(resolved))
            export_dense_hf_from_ckpt(ckpt, out / "hf", model=m)  # hfize: the dense model from the ckpt
            paths = {"quantized_dir": str(ckpt), "hf_dir": str(out / "hf")}
        payload["artifact_format"] = {"native": "quip_ckpt (unpacked Qidxs)", "hf": "huggingface_dense"}
    else:
        qcfg = ModelQuantConfig(bits=resolved.bits, group_size=resolved.group_size, iters=resolved.iters,
                                prior_tau=resolved.prior_tau, damping=resolved.damping,
                                polish_sweeps=resolved.polish_sweeps, polish_mode=resolved.polish_mode,
                                init=resolved.init, export_gptq=bool(resolved.save),
                                checkpoint_dir=str(out / "layers") if resume else None)
        res = quantize_model(m, ids, qcfg, group=group)
        payload["modules"] = {k: {kk: vv for kk, vv in v.items() if kk not in ("gptq", "q_int", "scale", "zero",
                                                                             "g_idx")}
                              for k, v in res["modules"].items()}
        if resolved.save and rank == 0:
            from .export import save_gptq_checkpoint
            save_gptq_checkpoint(m, res["modules"], out / "gptq", bits=resolved.bits, group_size=resolved.group_size,
                                 rotation="internal_hadamard")
            paths = {"quantized_dir": str(out / "gptq")}
        payload["artifact_format"] = {"native": "gptqmodel", "hf": "gptqmodel"}
    timings.update({f"quantize_{k}": float(v) for k, v in res["timings"].items()})
    timings["quantize"] = float(res["seconds"])
    timings["total"] = time.time() - t0
    payload.update(timings=timings, paths=paths, quant_time_s=float(res["seconds"]))
    if rank == 0:
        (out / "backend_results.json").write_text(json.dumps(payload, indent=2, sort_keys=True, default=str))
    return payload


__all__ = ["QuantizationConfig", "ResolvedQuantizationConfig", "SUPPORTED_BITS", "quantize"]
