"""LightX2V attention adapter for the b200_fp8 backend.

The reference ships an opt-in adapter that a LightX2V video DiT calls for every
self-attention layer (src/vc_attention/lightx2v.py:38-125).  It checks the call
layout, keeps one ``LayoutCache`` per generation, guards the layer/step order,
counts what the backend did and can capture the post-RoPE Q/K/V of chosen
layers and steps for offline replay.  Its MindIE arms target Ascend NPUs and
are not part of this package.  This module keeps the same contract on a B200:

* ``validate_layout`` accepts one dense, non-causal, unmasked self-attention
  sequence in SND or 1SND layout and returns BNSD views
  (lightx2v.py:18-35).
* ``ExperimentAdapter.apply`` takes the scheduler's step and the layer index
  from the call, starts a new cache generation when the scheduler's layout
  marker changes or layer ``l`` comes back at step 0, refuses repeated or
  reversed (layer, step) pairs, runs ``attention`` and returns ``[S, H*D]`` in
  the input dtype (lightx2v.py:48-96).
* With ``CaptureOptions`` it also saves the first heads of the post-RoPE
  Q/K/V of the chosen (rank, step, layer) calls, within a byte budget, as
  ``captures/rank{r}_step{s}_layer{l}.pt`` with the reference's metadata
  (lightx2v.py:92-125); ``error_report --capture`` replays such a file.
* ``configure`` checks and patches a LightX2V JSON config
  (lightx2v.py:128-144).
* ``main`` writes the patched config, registers the adapter with LightX2V's
  attention registry and runs ``lightx2v.infer`` (lightx2v.py:147-234).
  ``--prepare-only`` stops after writing the config.

LightX2V itself is imported only by ``main`` and ``register``.
"""
from __future__ import annotations

import argparse
import atexit
import json
import os
import runpy
import sys
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch

from .core import Config, LayoutCache, attention

# mode -> (v_smooth, expcast), the four arms of the reference (replay.py:17)
ARMS = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False),
        "combined": (True, True)}
REGISTRY_KEY = "b200_vc_attention"
_OPTIONS = {"scheduler", "block_idx", "causal", "softmax_scale", "dropout", "attn_mask", "mask", "pse"}


def validate_layout(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q, max_seqlen_kv, kwargs):
    """BNSD views of one dense self-attention sequence given as SND or 1SND;
    ``ValueError`` for anything the fused kernel would silently get wrong
    (lightx2v.py:18-35)."""
    unknown = sorted(set(kwargs) - _OPTIONS)
    if unknown:
        raise ValueError(f"Unknown attention options: {unknown}")
    if kwargs.get("causal", False) or kwargs.get("dropout", 0):
        raise ValueError("VC-Attention runs noncausal attention with dropout=0 only")
    for name in ("mask", "attn_mask", "pse"):
        if kwargs.get(name) is not None:
            raise ValueError(f"{name} is unsupported and would be ignored; refusing the call")
    if q.ndim == 4 and q.shape[0] == 1:
        q, k, v = (x[0] for x in (q, k, v))
    if any(x.ndim != 3 for x in (q, k, v)) or not (q.shape == k.shape == v.shape):
        raise ValueError("expected one dense self-attention sequence, SND or 1SND, with equal Q/K/V shapes")
    for cu, longest, length in ((cu_seqlens_q, max_seqlen_q, q.shape[0]),
                                (cu_seqlens_kv, max_seqlen_kv, k.shape[0])):
        if cu is not None and [int(x) for x in cu.tolist()] != [0, length]:
            raise ValueError("packed or multi-sequence attention is unsupported")
        if longest is not None and int(longest) != length:
            raise ValueError("max_seqlen does not match the single sequence")
    return [x.transpose(0, 1).unsqueeze(0) for x in (q, k, v)]


def _new_audit(mode):
    return {"mode": mode, "backend": "b200_fp8", "status": "running", "calls": 0, "smoothing_calls": 0,
            "regroup_calls": 0, "expcast_calls": 0, "captures": {}, "capture_bytes": 0}


@dataclass
class CaptureOptions:
    """Which attention calls to save and how much (the reference's
    --capture-* options and their defaults, lightx2v.py:153-158, :167)."""
    output_dir: str
    steps: tuple = (0, 4)
    layers: tuple = (0, 12)
    rank: int = 0
    heads: int = 1
    max_captures: int = 4
    max_capture_mib: int = 512
    model: str = "unspecified"
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if min(self.heads, self.max_captures, self.max_capture_mib) < 1:
            raise ValueError("capture heads, max-captures and max-capture-mib must be positive")


def capture(options, audit, q, k, v, *, step, steps, layer, scale, rank=None):
    """Save the first ``options.heads`` heads of BNSD post-RoPE Q/K/V for one
    (rank, step, layer) call, as the reference's ``_capture`` does
    (lightx2v.py:92-125): one file per key, at most ``max_captures`` files,
    and a ValueError rather than a silent skip when the byte budget would be
    exceeded.  Returns the path written, or None when the call is not
    selected."""
    rank = int(os.environ.get("RANK", "0")) if rank is None else rank
    if rank != options.rank or step not in options.steps or layer not in options.layers:
        return None
    key = f"rank{rank}_step{step}_layer{layer}"
    if key in audit["captures"] or len(audit["captures"]) >= options.max_captures:
        return None
    tensors = [x[:, :options.heads].detach() for x in (q, k, v)]
    nbytes = sum(x.numel() * x.element_size() for x in tensors)
    if audit["capture_bytes"] + nbytes > options.max_capture_mib * 1024 ** 2:
        raise ValueError("capture budget exceeded; capture fewer heads or calls, or raise max-capture-mib")
    target = Path(options.output_dir) / "captures" / f"{key}.pt"
    target.parent.mkdir(parents=True, exist_ok=True)
    metadata = {
        "model": options.model, "layout": "BNSD", "step": step, "total_steps": steps, "layer": layer,
        "rank": rank, "scale": scale, "full_shape": list(q.shape), "post_rope": True,
        "attention_boundary": "post_rope_and_optional_ulysses", "full_kv_context": True, "dtype": str(q.dtype),
        **options.extra,
    }
    torch.save({**dict(zip(("q", "k", "v"), (x.cpu().contiguous() for x in tensors))), "metadata": metadata},
               target)
    audit["captures"][key] = str(target.resolve())
    audit["capture_bytes"] += nbytes
    return target


class ExperimentAdapter:
    """Per-process attention hook for a LightX2V DiT (lightx2v.py:38-96).

    ``mode`` is one of ``ARMS``.  ``audit`` is a dict of counters that the
    launcher writes out at exit; ``attention_fn`` defaults to this package's
    ``attention`` (tests pass a stand-in); ``capture`` (CaptureOptions) saves
    the selected calls' Q/K/V before they are attended."""

    def __init__(self, mode, audit=None, *, attention_fn=None, capture=None):
        if mode not in ARMS:
            raise ValueError(f"mode must be one of {sorted(ARMS)}")
        smooth, cast = ARMS[mode]
        self.mode = mode
        self.audit = _new_audit(mode) if audit is None else audit
        self.capture_options = capture
        self.vc_config = Config(v_smooth=smooth, expcast=cast)
        self.cache = LayoutCache(self.vc_config)
        self._attention = attention_fn or attention
        self._marker = None
        self._generation = 0
        self._last_steps = {}

    def _track(self, scheduler, layer):
        """Cache generation and (layer, step) order (lightx2v.py:53-68)."""
        marker = getattr(scheduler, "layout_cpu", None)
        if marker is None:
            raise ValueError("scheduler.layout_cpu is missing: this adapter needs the DiT scheduler's "
                             "per-request layout marker")
        step, steps = int(scheduler.step_index), int(scheduler.infer_steps)
        if marker is not self._marker or (step == 0 and layer in self._last_steps):
            # a new request: drop every cached layout; keep the marker itself
            # alive so that a recycled id() can never look like the old one
            self.cache.reset()
            self._marker = marker
            self._generation += 1
            self._last_steps.clear()
        last = self._last_steps.get(layer)
        if last is not None and step <= last:
            raise ValueError(f"layer {layer} called again at step {step} after step {last}: repeated or "
                             "reversed calls (head-parallel, CFG, re-entry) are unsupported")
        self._last_steps[layer] = step
        return step, steps

    @torch.no_grad()
    def apply(self, q, k, v, cu_seqlens_q=None, cu_seqlens_kv=None, max_seqlen_q=None, max_seqlen_kv=None,
              **kwargs):
        q4, k4, v4 = validate_layout(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q, max_seqlen_kv, kwargs)
        scheduler, layer = kwargs.get("scheduler"), kwargs.get("block_idx")
        if scheduler is None or layer is None:
            raise ValueError("scheduler and block_idx are required; route attention calls without them "
                             "(the refiner) to another attention type")
        step, steps = self._track(scheduler, layer)
        scale = kwargs.get("softmax_scale")
        scale = q4.shape[-1] ** -0.5 if scale is None else scale
        self.audit["calls"] += 1
        if self.capture_options is not None:
            capture(self.capture_options, self.audit, q4, k4, v4, step=step, steps=steps, layer=layer, scale=scale)
        out, stats = self._attention(q4, k4, v4, self.vc_config, cache=self.cache, step=step, total_steps=steps,
                                     request_id=self._generation, layer_id=layer, scale=scale)
        self.audit["smoothing_calls"] += int(bool(stats["smoothing_active"]))
        self.audit["regroup_calls"] += int(bool(stats["layout_refreshed"]))
        self.audit["expcast_calls"] += int(bool(stats["expcast"]))
        s, h = q4.shape[2], q4.shape[1]
        return out[0].transpose(0, 1).reshape(s, h * out.shape[-1]).to(q.dtype)


def configure(base):
    """Checked copy of a LightX2V config with attention routed to this
    adapter (lightx2v.py:128-144)."""
    config = dict(base)
    parallel = config.get("parallel", {}) or {}
    if config.get("use_compile", False):
        raise ValueError("use_compile must be off: the adapter is an eager attention call")
    if config.get("warmup", False):
        raise ValueError("warmup must be off: warm-up tensors would start a layout generation")
    if parallel.get("seq_p_head_parallel", False):
        raise ValueError("seq_p_head_parallel must be off: head identity is not passed to the adapter")
    if parallel.get("seq_p_attn_type", "ulysses") != "ulysses":
        raise ValueError("only Ulysses sequence parallelism is supported (each rank sees whole heads)")
    if config.get("enable_cfg", False):
        raise ValueError("CFG is unsupported: its second pass repeats each (layer, step)")
    config["warmup"] = False
    config["attn_type"] = REGISTRY_KEY
    return config


def register(registry, template, mode, audit, capture_options=None):
    """Register the adapter class under ``REGISTRY_KEY`` with LightX2V's
    attention registry (``ATTN_WEIGHT_REGISTER``), mixed with its template
    base class (lightx2v.py:203-207)."""

    class RegisteredAdapter(ExperimentAdapter, template):
        def __init__(self):
            ExperimentAdapter.__init__(self, mode, audit, capture=capture_options)

    registry.register(RegisteredAdapter, key=REGISTRY_KEY)
    return RegisteredAdapter


def main(argv=None):
    parser = argparse.ArgumentParser(description="Run LightX2V inference with VC-Attention on B200")
    parser.add_argument("--mode", choices=sorted(ARMS), required=True)
    parser.add_argument("--output-dir", required=True)
    parser.add_argument("--prepare-only", action="store_true",
                        help="write the patched config and stop (no LightX2V import)")
    parser.add_argument("--capture", action="store_true",
                        help="also save post-RoPE Q/K/V of the selected calls under OUTPUT_DIR/captures")
    parser.add_argument("--capture-steps", type=int, nargs="+", default=[0, 4])
    parser.add_argument("--capture-layers", type=int, nargs="+", default=[0, 12])
    parser.add_argument("--capture-rank", type=int, default=0)
    parser.add_argument("--capture-heads", type=int, default=1)
    parser.add_argument("--max-captures", type=int, default=4)
    parser.add_argument("--max-capture-mib", type=int, default=512)
    parser.add_argument("lightx_args", nargs=argparse.REMAINDER)
    options = parser.parse_args(argv)
    capture_options = None
    if options.capture:
        try:
            capture_options = CaptureOptions(
                output_dir=options.output_dir, steps=tuple(options.capture_steps),
                layers=tuple(options.capture_layers), rank=options.capture_rank, heads=options.capture_heads,
                max_captures=options.max_captures, max_capture_mib=options.max_capture_mib)
        except ValueError as exc:
            parser.error(str(exc))
    args = list(options.lightx_args)
    if args[:1] == ["--"]:
        args = args[1:]
    if "--config_json" not in args or args.index("--config_json") + 1 >= len(args):
        parser.error("pass the LightX2V arguments after --, including --config_json PATH")
    index = args.index("--config_json") + 1
    source = Path(args[index])
    config = configure(json.loads(source.read_text(encoding="utf-8")))
    out = Path(options.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    rank = int(os.environ.get("RANK", "0"))
    patched = out / f"config.rank{rank}.json"
    patched.write_text(json.dumps(config, indent=2) + "\n", encoding="utf-8")
    args[index] = str(patched.resolve())
    if options.prepare_only:
        print(patched.resolve())
        return 0

    from lightx2v.utils.registry_factory import ATTN_WEIGHT_REGISTER
    from lightx2v_platform.ops.attn.template import AttnWeightTemplate

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    audit = _new_audit(options.mode)
    audit.update(rank=rank, argv=args, source_config=str(source.resolve()),
                 vc_config=asdict(Config(v_smooth=ARMS[options.mode][0], expcast=ARMS[options.mode][1])))
    register(ATTN_WEIGHT_REGISTER, AttnWeightTemplate, options.mode, audit, capture_options)

    def save_audit():
        (out / f"audit.rank{rank}.json").write_text(json.dumps(audit, indent=2) + "\n", encoding="utf-8")

    atexit.register(save_audit)
    sys.argv = ["lightx2v.infer", *args]
    try:
        runpy.run_module("lightx2v.infer", run_name="__main__")
    except BaseException:
        audit["status"] = "failed"
        raise
    else:
        if audit["calls"] == 0:
            audit["status"] = "failed_no_attention_calls"
            raise RuntimeError("LightX2V ran but no attention call reached the adapter")
        audit["status"] = "completed"
    finally:
        save_audit()
    return 0


if __name__ == "__main__":
    sys.exit(main())
