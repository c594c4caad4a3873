"""Calibration on CUDA: running per-(head, frequency) query sums and the model driver.

``LayerAccumulator.add`` has the contract of the reference's stats builder
(src/vllm_ascend_kvcompress/calibration.py:87-131, ``_LayerAccumulator``): it
takes one forward's pre-RoPE query projection, accepts the packed
query+gate layout and the [..., heads, head_dim] layout, and accumulates the
sums of the real part q[:F], the imaginary part q[F:rot], the modulus and the
unrotated dims q[rot:], plus the row count.  The sums run in
``kvc_calibration_accumulate`` and stay on the device in fp64 until ``means``.

The driver (``generate_calibration_artifact``, ``ensure_calibration_for_runner``,
``main``) follows the reference's calibration.py:134-748: load the Hugging Face
model on CUDA, hook every full-attention layer's ``q_norm`` (else ``q_proj``),
run one forward over the calibration text, and write the schema-3 artefact
(same fields, same metadata, same validation, written atomically under a file
lock).  Differences: the reduction runs on the GPU in fp64 (the reference sums
fp32 on the host); the device must be CUDA and the model bfloat16 or float16
(the kernel's input types); the built-in calibration text is this package's own
(label ``builtin:b200-systems-v1``), so artefacts generated without an input
file are not byte-identical to the reference's — with the same input file the
statistics agree within the calibration tolerance.
"""

from __future__ import annotations

import argparse
import fcntl
import gc
import hashlib
import importlib.util
import json
import os
import tempfile
from collections.abc import Mapping, Sequence
from contextlib import suppress
from dataclasses import dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

import torch

from . import __version__
from .methods.base import ModelShape
from .methods.triattention import kernels as K
from .methods.triattention.config import TriAttentionConfig
from .methods.triattention.stats import SUPPORTED_MODEL_TYPES, CalibrationStats
from .model import model_shape_from_config

GENERATOR = "vllm-ascend-kvcompress-hust"  # artefact generator name (the serving-time checks key on it)
BUILTIN_INPUT_SOURCE = "builtin:b200-systems-v1"


class LayerAccumulator:
    """Online calibration sums of one attention layer."""

    def __init__(self) -> None:
        self.real_sum: torch.Tensor | None = None
        self.imag_sum: torch.Tensor | None = None
        self.abs_sum: torch.Tensor | None = None
        self.pass_sum: torch.Tensor | None = None
        self.count = 0
        self._ws: torch.Tensor | None = None

    def add(self, projected: torch.Tensor, heads: int, head_dim: int, rotary_dim: int, *,
            first_position: int | None = None, omega: torch.Tensor | None = None) -> None:
        """Add one batch of query rows.

        Pre-RoPE projections by default (the stats builder's input).  With
        ``first_position`` and ``omega`` the rows are post-RoPE attention inputs
        at positions ``first_position + t``; the reduction undoes the rotation
        in fp32 before summing.
        """
        expected = heads * head_dim
        if projected.shape[-1] == expected * 2:
            projected = projected[..., :expected]  # Qwen3.5 packs the output gate after Q
        if projected.shape[-1] == expected:
            rows = projected.detach().reshape(-1, expected)
        elif projected.shape[-1] == head_dim and projected.numel() % expected == 0:
            rows = projected.detach().reshape(-1, expected)
        else:
            raise RuntimeError("query projection width does not match model attention shape: "
                               f"got {projected.shape[-1]}, expected {expected}")
        K.require_cuda(rows)
        if rows.stride(-1) != 1:
            rows = rows.contiguous()
        if rows.dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError("calibration queries must be bfloat16 or float16 on the CUDA path")
        f = rotary_dim // 2
        p = head_dim - rotary_dim
        dev = rows.device
        if self.real_sum is None:
            z = lambda w: torch.zeros(heads, w, dtype=torch.float64, device=dev)
            self.real_sum, self.imag_sum, self.abs_sum = z(f), z(f), z(f)
            self.pass_sum = z(p) if p else None
        need = K.calibration_workspace_doubles(rows.shape[0], heads, head_dim, rotary_dim)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.float64, device=dev)
        K.calibration_accumulate(rows, heads, head_dim, rotary_dim, self.real_sum, self.imag_sum, self.abs_sum,
                                 self.pass_sum, self._ws, first_position=first_position, omega=omega)
        self.count += rows.shape[0]

    def means(self) -> dict[str, torch.Tensor]:
        """fp32 CPU means in the schema-3 ``layer_stats`` field names."""
        if self.count <= 0 or self.real_sum is None:
            raise RuntimeError("no query values captured for this layer")
        d = float(self.count)
        out = {
            "q_mean_real": (self.real_sum / d).float().cpu(),
            "q_mean_imag": (self.imag_sum / d).float().cpu(),
            "q_abs_mean": (self.abs_sum / d).float().cpu(),
        }
        if self.pass_sum is not None:
            out["q_pass_mean"] = (self.pass_sum / d).float().cpu()
        return out


_LayerAccumulator = LayerAccumulator  # the reference's private name

# Plain-prose calibration text written for this package (used when no input file is given).
_BUILTIN_SECTIONS = (
    """The maintenance crew inspected the pumping station at dawn. Two of the four
pumps ran within their rated range, a third showed a slow pressure decay of about
one percent per hour, and the fourth was isolated for a bearing replacement. The
log records each reading with its unit, the time it was taken and who took it.""",
    """A library catalogue keeps one record per edition. Each record lists the
title, the authors in the order printed on the cover, the publisher, the year,
the number of pages and a shelf mark. When two copies of an edition differ, the
note field says how: a missing map, a later binding, a signature on the flyleaf.""",
    """To convert a recipe for four people into one for six, multiply every
quantity by one and a half, then round to amounts that can be measured: 300 g of
flour becomes 450 g, two eggs become three, and 250 ml of milk becomes 375 ml.
Baking time changes less than the quantities, so check the oven after the time
given in the original recipe.""",
    """Un tren sale de la estacion a las nueve y diez y llega a la costa a las
once y cuarenta. Der Zug hält zweimal, einmal an einer Brücke und einmal in einem
kleinen Dorf. Le contrôleur vérifie les billets entre les deux arrêts, et les
passagers notent l'heure exacte de chaque arrivée.""",
    """def moving_average(values, window):
    total = sum(values[:window])
    out = [total / window]
    for i in range(window, len(values)):
        total += values[i] - values[i - window]
        out.append(total / window)
    return out
The function above keeps a running sum, so each new average costs two additions
instead of a full pass over the window.""",
)


@dataclass(frozen=True)
class CalibrationRequest:
    """One artefact to generate (fields as the reference's CalibrationRequest, calibration.py:69-84)."""

    model: str
    output: Path
    input_path: Path | None = None
    tokenizer: str | None = None
    revision: str | None = None
    tokenizer_revision: str | None = None
    trust_remote_code: bool = False
    local_files_only: bool = False
    max_length: int = 4096
    device: str = "cuda"
    device_map: str | None = None
    dtype: str = "bfloat16"
    attn_implementation: str = "eager"
    force: bool = False


def ensure_calibration_for_runner(runner: Any, selection: Any) -> bool:
    """Generate (when missing and allowed) and validate the artefact before serving weights load.

    Mirrors calibration.py:134-177: only for the triattention method; an
    existing artefact is validated; a missing one is generated when
    ``auto_calibrate`` is on, with the runner's model, tokenizer, revision,
    dtype and device ("auto" = the runner's device), spreading the model over
    the visible GPUs (``device_map="auto"``) when serving is tensor parallel.
    """
    if getattr(selection, "method", None) != "triattention":
        return False
    config = TriAttentionConfig.from_method_config(selection.method_config)
    model_config = runner.model_config
    shape = model_shape_from_config(model_config)
    if config.stats_path.is_file():
        _validate_artifact(config.stats_path, shape, model_config)
        return False
    if not config.auto_calibrate:
        return False
    device = str(getattr(runner, "device", "cuda")) if config.calibration_device == "auto" else \
        config.calibration_device
    parallel = getattr(getattr(runner, "vllm_config", None), "parallel_config", None)
    tp = int(getattr(parallel, "tensor_parallel_size", 1))
    request = CalibrationRequest(
        model=str(model_config.model),
        tokenizer=str(model_config.tokenizer) if getattr(model_config, "tokenizer", None) else None,
        output=config.stats_path,
        input_path=config.calibration_input_path,
        revision=getattr(model_config, "revision", None),
        tokenizer_revision=getattr(model_config, "tokenizer_revision", None),
        trust_remote_code=bool(getattr(model_config, "trust_remote_code", False)),
        local_files_only=config.calibration_local_files_only,
        max_length=config.calibration_max_length,
        device=device,
        device_map="auto" if tp > 1 else None,
        dtype=_dtype_name(getattr(model_config, "dtype", "bfloat16")),
        attn_implementation=config.calibration_attn_implementation,
    )
    generated = generate_calibration_artifact(request)
    _validate_artifact(config.stats_path, shape, model_config)
    return generated


def generate_calibration_artifact(request: CalibrationRequest) -> bool:
    """Write one artefact; False when it already exists (another process won the race) and force is off."""
    if request.max_length < 128:
        raise ValueError("calibration max_length must be at least 128")
    output = request.output.expanduser().resolve()
    output.parent.mkdir(parents=True, exist_ok=True)
    lock = output.with_name(f".{output.name}.lock")
    with lock.open("a+b") as handle:
        fcntl.flock(handle.fileno(), fcntl.LOCK_EX)
        if output.is_file() and not request.force:
            _validate_existing_for_request(output, request)
            return False
        payload = _generate_payload(request)
        _atomic_torch_save(payload, output)
    return True


def _cuda_device(request: CalibrationRequest) -> torch.device:
    device = torch.device(request.device)
    if device.type != "cuda":
        raise RuntimeError(f"the B200 calibration driver reduces on CUDA; got device {request.device!r}")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available; the B200 calibration driver has no CPU path")
    if request.device_map is not None and importlib.util.find_spec("accelerate") is None:
        raise RuntimeError("device_map='auto' calibration requires the Accelerate package")
    return torch.device("cuda", torch.cuda.current_device() if device.index is None else device.index)


def _generate_payload(request: CalibrationRequest) -> dict[str, Any]:
    device = _cuda_device(request)
    dtype = _torch_dtype(request.dtype)
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the CUDA calibration reduction takes bfloat16 or float16 query projections")
    try:
        from transformers import AutoConfig, AutoModel, AutoModelForCausalLM, AutoTokenizer
        from transformers import __version__ as transformers_version
    except ImportError as error:
        raise RuntimeError("calibration generation requires the Transformers package") from error
    common = {"trust_remote_code": request.trust_remote_code, "local_files_only": request.local_files_only}
    config = AutoConfig.from_pretrained(request.model, revision=request.revision, **common)
    shape = _model_shape_from_hf_config(config)
    if shape.model_type not in SUPPORTED_MODEL_TYPES:
        raise ValueError(f"model_type {shape.model_type!r} is not supported for calibration")
    tokenizer_id = request.tokenizer or request.model
    tokenizer = AutoTokenizer.from_pretrained(tokenizer_id, revision=request.tokenizer_revision or request.revision,
                                              **common)
    text, source = _load_calibration_text(request)
    encoded = tokenizer(text, return_tensors="pt", truncation=True, max_length=request.max_length,
                        add_special_tokens=True)
    ids = encoded.get("input_ids")
    if not isinstance(ids, torch.Tensor) or ids.ndim != 2:
        raise RuntimeError("tokenizer did not return rank-two input_ids")
    token_count = int(ids.shape[1])
    if token_count < 2:
        raise ValueError("calibration input produced fewer than two tokens")
    text_config = getattr(config, "text_config", config)
    nested = text_config is not config and str(getattr(config, "model_type", "")).startswith("qwen3_5")
    options: dict[str, Any] = {"config": text_config if nested else config, "revision": request.revision,
                               "dtype": dtype, **common}
    if request.device_map is not None:  # placement by Accelerate; else load, then move to the device
        options["device_map"] = request.device_map
    if request.attn_implementation:
        options["attn_implementation"] = request.attn_implementation
    if nested:  # Qwen3.5 keeps the text weights under model.language_model
        options["key_mapping"] = {r"^model\.language_model\.(.+)$": r"model.\1"}
    model = None
    hooks: list[Any] = []
    try:
        model = (AutoModelForCausalLM if nested else AutoModel).from_pretrained(request.model, **options)
        if request.device_map is None:
            model.to(device)
        model.eval()
        layers = _find_attention_layers(model)
        found = tuple(i for i, _ in layers)
        if found != shape.full_attention_layer_indices:
            raise RuntimeError("located full-attention layers do not match model config: "
                               f"got {found}, expected {shape.full_attention_layer_indices}")
        sums = {i: LayerAccumulator() for i, _ in layers}
        for i, attention in layers:
            target = getattr(attention, "q_norm", None)
            if not isinstance(target, torch.nn.Module):
                target = getattr(attention, "q_proj", None)
            if not isinstance(target, torch.nn.Module):
                raise RuntimeError(f"attention layer {i} exposes neither q_norm nor q_proj")
            hooks.append(target.register_forward_hook(_capture_hook(sums[i], i, shape)))
        inputs_device = torch.device("cpu") if request.device_map == "auto" else device
        inputs = {k: v.to(inputs_device) for k, v in encoded.items() if isinstance(v, torch.Tensor)}
        with torch.inference_mode():
            model(**inputs, use_cache=False)
        rope_type = _rope_type(config)
        rope = _extract_rope_values(model, layers, shape, rope_type)
        layer_stats: dict[str, dict[str, torch.Tensor]] = {}
        for i, acc in sums.items():
            values = acc.means()
            inv_freq, freq_scale_sq = rope[i]
            values["inv_freq"] = inv_freq
            values["freq_scale_sq"] = freq_scale_sq
            layer_stats[str(i)] = {k: v.contiguous() for k, v in values.items()}
        config_dict = config.to_dict() if hasattr(config, "to_dict") else vars(config)
        metadata = {
            "schema_version": 3,
            "generator": GENERATOR,
            "generator_version": __version__,
            "transformers_version": transformers_version,
            "created_at_utc": datetime.now(timezone.utc).isoformat(),
            "model": request.model,
            "model_revision": request.revision or "default",
            "model_source_fingerprint": _model_source_fingerprint(request.model, request.revision),
            "tokenizer": tokenizer_id,
            "tokenizer_revision": request.tokenizer_revision or request.revision or "default",
            "model_config_sha256": _sha256_json(config_dict),
            "input_source": source,
            "input_sha256": hashlib.sha256(text.encode("utf-8")).hexdigest(),
            "token_count": token_count,
            "requested_max_length": request.max_length,
            "num_traces": 1,
            "model_type": shape.model_type,
            "num_layers": shape.num_layers,
            "num_attention_heads": shape.num_attention_heads,
            "num_kv_heads": shape.num_kv_heads,
            "head_dim": shape.head_dim,
            "rotary_dim": shape.effective_rotary_dim,
            "attention_layer_indices": list(shape.full_attention_layer_indices),
            "rope_theta": shape.rope_theta,
            "rope_style": "half",
            "rope_type": rope_type,
            "dtype": request.dtype,
            "attn_implementation": request.attn_implementation,
        }
        payload = {"metadata": metadata, "layer_stats": layer_stats}
        reasons = _load_payload(payload).validate(shape)
        if reasons:
            raise ValueError("generated calibration is incompatible: " + "; ".join(reasons))
        return payload
    finally:
        for hook in hooks:
            hook.remove()
        del model
        gc.collect()
        _empty_device_cache(request.device_map == "auto")


def _capture_hook(acc: LayerAccumulator, index: int, shape: ModelShape):
    def capture(_module: torch.nn.Module, _inputs: tuple[Any, ...], output: Any) -> None:
        if not isinstance(output, torch.Tensor):
            raise RuntimeError(f"attention layer {index} q_proj returned a non-tensor")
        acc.add(output, shape.num_attention_heads, shape.head_dim, shape.effective_rotary_dim)

    return capture


def _load_payload(payload: Mapping[str, Any]) -> CalibrationStats:
    """Round-trip a payload through the artefact loader so it gets the same validation."""
    fd, name = tempfile.mkstemp(suffix=".pt")
    os.close(fd)
    path = Path(name)
    try:
        torch.save(dict(payload), path)
        return CalibrationStats.load(path)
    finally:
        path.unlink(missing_ok=True)


def _validate_artifact(path: Path, shape: ModelShape, model_config: Any | None = None) -> None:
    artefact = CalibrationStats.load(path)
    reasons = list(artefact.validate(shape))
    if model_config is not None and artefact.metadata.get("generator") == GENERATOR:
        model = str(model_config.model)
        revision = getattr(model_config, "revision", None)
        expected = {"model": model, "model_revision": revision or "default",
                    "model_source_fingerprint": _model_source_fingerprint(model, revision)}
        for key, want in expected.items():
            got = artefact.metadata.get(key)
            if got != want:
                reasons.append(f"calibration {key} {got!r} does not match {want!r}")
    if reasons:
        raise ValueError(f"calibration artifact {path} is incompatible: " + "; ".join(reasons))


def _validate_existing_for_request(path: Path, request: CalibrationRequest) -> None:
    try:
        from transformers import AutoConfig
    except ImportError as error:
        raise RuntimeError("calibration validation requires the Transformers package") from error
    config = AutoConfig.from_pretrained(request.model, revision=request.revision,
                                        trust_remote_code=request.trust_remote_code,
                                        local_files_only=request.local_files_only)
    model_config = type("ModelConfig", (), {"model": request.model, "revision": request.revision})()
    _validate_artifact(path, _model_shape_from_hf_config(config), model_config)


def _atomic_torch_save(payload: Mapping[str, Any], output: Path) -> None:
    fd, name = tempfile.mkstemp(prefix=f".{output.name}.", suffix=".tmp", dir=output.parent)
    tmp = Path(name)
    try:
        with os.fdopen(fd, "wb") as stream:
            torch.save(dict(payload), stream)
            stream.flush()
            os.fsync(stream.fileno())
        os.replace(tmp, output)
    except BaseException:
        with suppress(OSError):
            os.close(fd)
        tmp.unlink(missing_ok=True)
        raise


def _find_transformer_backbone(model: torch.nn.Module) -> torch.nn.Module:
    """Breadth-first search through model / language_model / text_model for the decoder layer list."""
    queue, seen = [model], set()
    while queue:
        node = queue.pop(0)
        if id(node) in seen:
            continue
        seen.add(id(node))
        if isinstance(getattr(node, "layers", None), torch.nn.ModuleList):
            return node
        for name in ("model", "language_model", "text_model"):
            child = getattr(node, name, None)
            if isinstance(child, torch.nn.Module):
                queue.append(child)
    raise RuntimeError("cannot locate transformer decoder layers")


def _find_attention_layers(model: torch.nn.Module) -> list[tuple[int, torch.nn.Module]]:
    layers = _find_transformer_backbone(model).layers
    return [(i, layer.self_attn) for i, layer in enumerate(layers)
            if isinstance(getattr(layer, "self_attn", None), torch.nn.Module)]


def _extract_rope_values(model: torch.nn.Module, layers: Sequence[tuple[int, torch.nn.Module]], shape: ModelShape,
                         rope_type: str) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
    """(inv_freq [F], freq_scale_sq [1, F]) per layer, from the model's rotary module(s)."""
    shared = getattr(_find_transformer_backbone(model), "rotary_emb", None)
    rot = shape.effective_rotary_dim
    F = rot // 2
    out = {}
    for i, attention in layers:
        rotary = getattr(attention, "rotary_emb", shared)
        inv_freq = getattr(rotary, "inv_freq", None)
        if isinstance(inv_freq, torch.Tensor):
            inv_freq = inv_freq.detach().float().cpu().flatten()
        elif rope_type == "default":
            inv_freq = 1.0 / (shape.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
        else:
            raise RuntimeError(f"scaled RoPE layer {i} does not expose exact inv_freq")
        if inv_freq.numel() != F:
            raise RuntimeError(f"layer {i} inv_freq has {inv_freq.numel()} values; expected {F}")
        scale = torch.as_tensor(getattr(rotary, "attention_scaling", 1.0), dtype=torch.float32).cpu().flatten()
        if scale.numel() == 1:
            scale = scale.expand(F)
        elif scale.numel() in (shape.head_dim, rot):
            scale = scale[:F]
        elif scale.numel() != F:
            raise RuntimeError(f"layer {i} attention scaling has {scale.numel()} values")
        out[i] = (inv_freq.contiguous(), scale.square().unsqueeze(0).contiguous())
    return out


def _model_shape_from_hf_config(config: Any) -> ModelShape:
    return model_shape_from_config(type("ModelConfig", (), {"hf_text_config": getattr(config, "text_config",
                                                                                         config)})())


def _rope_type(config: Any) -> str:
    config = getattr(config, "text_config", config)
    params = getattr(config, "rope_parameters", None)
    raw = params if isinstance(params, Mapping) else getattr(config, "rope_scaling", None)
    if isinstance(raw, Mapping):
        return str(raw.get("rope_type", raw.get("type", "default")) or "default")
    return "default"


def _load_calibration_text(request: CalibrationRequest) -> tuple[str, str]:
    """(text, source label): the input file, else the built-in sections repeated to ~6 characters per token."""
    if request.input_path is not None:
        path = request.input_path.expanduser().resolve()
        if not path.is_file():
            raise ValueError(f"calibration input file does not exist: {path}")
        text = path.read_text(encoding="utf-8")
        if not text.strip():
            raise ValueError(f"calibration input file is empty: {path}")
        return text, str(path)
    want = request.max_length * 6
    parts, size, rnd = [], 0, 1
    while size < want:
        for j, section in enumerate(_BUILTIN_SECTIONS, 1):
            block = f"Part {rnd}.{j}\n{section}\n"
            parts.append(block)
            size += len(block)
        rnd += 1
    return "\n".join(parts), BUILTIN_INPUT_SOURCE


def _empty_device_cache(all_devices: bool) -> None:
    if not torch.cuda.is_available():
        return
    for index in (range(torch.cuda.device_count()) if all_devices else (torch.cuda.current_device(),)):
        with torch.cuda.device(index):
            torch.cuda.empty_cache()


def _torch_dtype(value: str) -> torch.dtype:
    table = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
    name = _dtype_name(value)
    if name not in table:
        raise ValueError(f"unsupported calibration dtype: {value}")
    return table[name]


def _dtype_name(value: Any) -> str:
    name = str(value).replace("torch.", "").lower()
    return {"half": "float16", "float": "float32", "auto": "bfloat16"}.get(name, name)


def _sha256_json(value: Any) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"), default=str).encode()).hexdigest()


def _model_source_fingerprint(model: str, revision: str | None) -> str:
    """A local checkpoint's manifest (names, sizes, mtimes) hashed, else the identifier@revision hashed."""
    path = Path(model).expanduser()
    if not path.is_dir():
        return "identifier:" + hashlib.sha256(f"{model}@{revision or 'default'}".encode()).hexdigest()
    files = sorted({f for pat in ("*.safetensors", "*.bin", "*.pt", "*.index.json", "config.json")
                    for f in path.glob(pat) if f.is_file()})
    if not files:
        raise ValueError(f"model directory contains no recognized checkpoint files: {path}")
    return "local-manifest:" + _sha256_json([(str(f.relative_to(path)), int(f.stat().st_size),
                                              int(f.stat().st_mtime_ns)) for f in files])


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Generate model-matched TriAttention calibration statistics (CUDA).")
    p.add_argument("--model", required=True)
    p.add_argument("--output", required=True, type=Path)
    p.add_argument("--input", dest="input_path", type=Path)
    p.add_argument("--tokenizer")
    p.add_argument("--revision")
    p.add_argument("--tokenizer-revision")
    p.add_argument("--max-length", type=int, default=4096)
    p.add_argument("--device", default="cuda")
    p.add_argument("--device-map", choices=("auto",),
                   help="spread a large temporary calibration model over the visible GPUs")
    p.add_argument("--dtype", choices=("float16", "bfloat16"), default="bfloat16")
    p.add_argument("--attn-implementation", choices=("eager", "sdpa", "flash_attention_2"), default="eager")
    p.add_argument("--trust-remote-code", action="store_true")
    p.add_argument("--local-files-only", action="store_true")
    p.add_argument("--force", action="store_true")
    return p


def request_from_args(argv: Sequence[str] | None = None) -> CalibrationRequest:
    a = _build_parser().parse_args(argv)
    return CalibrationRequest(model=a.model, output=a.output, input_path=a.input_path, tokenizer=a.tokenizer,
                              revision=a.revision, tokenizer_revision=a.tokenizer_revision,
                              trust_remote_code=a.trust_remote_code, local_files_only=a.local_files_only,
                              max_length=a.max_length, device=a.device, device_map=a.device_map, dtype=a.dtype,
                              attn_implementation=a.attn_implementation, force=a.force)


def main(argv: Sequence[str] | None = None) -> int:
    request = request_from_args(argv)
    generated = generate_calibration_artifact(request)
    print(f"{'generated' if generated else 'reused'} calibration artifact: {request.output}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
