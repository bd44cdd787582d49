"""Model construction from training arguments and checkpoint payloads.

``build_model(rules, num_xfers, args)`` mirrors the reference's
``model_factory.build_model`` (model_factory.py:7-41) for the paged action
architecture: the same argument names and defaults.  ``load_checkpoint``
reads the payload the reference's trainer saves, ``{"model": state_dict,
"args": vars(args), "metrics": ..., "format": ...}`` (train.py:482-490), and
loads it the way the search does (paged_rollout_benchmark.py:707-714):
build from ``payload["args"]``, load the state dict, switch the readout to
the paged backend.  Parameter names and shapes are the reference's, so the
state dict loads unchanged.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

from .paged_model import PagedActionBindingModel
from .synthetic import RuleMetadata


def build_model(rules: RuleMetadata, num_xfers: int, args: dict,
                compute_dtype: torch.dtype = torch.bfloat16) -> PagedActionBindingModel:
    """The reference's argument mapping (model_factory.py:7-41).  Only the
    ``paged_action`` architecture runs the decode path; the legacy
    ``S0ActionBindingModel`` (full-history recompute) is not part of it."""
    architecture = args.get("architecture", "legacy")
    if architecture != "paged_action":
        raise NotImplementedError(
            f"architecture {architecture!r}: the B200 decode path runs the paged action model "
            "(architecture 'paged_action')")
    backend = args.get("readout_attention_backend", "sdpa")
    if backend not in ("eager", "sdpa", "sdpa_live", "paged"):
        raise ValueError(f"unknown readout attention backend: {backend}")
    return PagedActionBindingModel(
        rules,
        num_xfers=num_xfers,
        width=args["width"],
        retrieval_width=args["retrieval_width"],
        graph_layers=args["graph_layers"],
        action_layers=args.get("action_layers", 4),
        action_heads=args.get("action_heads", 6),
        max_sequence_length=args.get("max_sequence_length", 256),
        ordered_binding_roles=args.get("ordered_binding_roles", False),
        readout_graph_layers=args.get("readout_graph_layers", 0),
        readout_graph_input=args.get("readout_graph_input", "cached"),
        readout_locality_features=args.get("readout_locality_features", False),
        identity_readout_prefix=args.get("identity_readout_prefix", 0),
        # every backend computes the same readout; this one reads the paged
        # readout K/V in place (the search sets the attribute the same way)
        readout_attention_backend="paged",
        dropout=0.0,
        compute_dtype=compute_dtype,
    )


def load_checkpoint(source: str | Path | dict[str, Any], rules: RuleMetadata, *,
                    device: torch.device | str = "cuda",
                    compute_dtype: torch.dtype = torch.bfloat16) -> PagedActionBindingModel:
    """A trained model from the trainer's checkpoint payload (a path to the
    ``torch.save`` file or the loaded dict), in eval mode on `device`."""
    payload = source if isinstance(source, dict) else torch.load(
        Path(source), map_location="cpu", weights_only=False)
    missing = [k for k in ("model", "args") if k not in payload]
    if missing:
        raise ValueError(f"checkpoint payload lacks {missing}: expected the trainer's "
                         "{'model', 'args', 'metrics', 'format'} dictionary")
    model = build_model(rules, rules.num_xfers, payload["args"], compute_dtype)
    model.load_state_dict(payload["model"])
    return model.to(device).eval()
