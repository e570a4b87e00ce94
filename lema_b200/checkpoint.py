"""Weights into and out of the streamed trainer's int8 segments.

* ``HFCheckpoint``: an index over a Hugging Face safetensors checkpoint (one file
  or a directory of shards), the files the reference's ``GlobalBinaryIndex``
  reads (src/lema/_gbi.py:9-31) under the parameter names its adapters request
  (src/lema/adapters/_llama.py:41-57, _mixtral.py:50-68). ``pack_block_from_hf``
  quantises one block's projection weights per output channel on the device (K1)
  and writes them, the norms and (MoE) the experts and router, into the block's
  segment.
* int8 segment files: ``save_segments`` writes every block's packed segment as
  one uint8 tensor [blocks, segment bytes] plus the embedding, final norm and
  lm_head, with the model shape and the segment layout in the safetensors
  metadata; ``load_segments`` checks both and copies the bytes straight into the
  pinned segments (each rank of a sharded stream reads only its chunk). A
  pre-quantised checkpoint therefore loads without touching a float weight.
"""
from __future__ import annotations

import dataclasses
import glob
import json
import os

import torch

from . import ops

SEGMENT_FORMAT = "lema_b200.w8a8-segments.v1"

_ATTN = ("q_proj", "k_proj", "v_proj", "o_proj")
_MLP = ("gate_proj", "up_proj", "down_proj")


class HFCheckpoint:
    """Name -> tensor over the safetensors files of a checkpoint."""

    def __init__(self, path: str):
        from safetensors import safe_open
        if os.path.isdir(path):
            files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        else:
            files = [path]
        if not files or not all(os.path.exists(f) for f in files):
            raise FileNotFoundError(f"no .safetensors files at {path}")
        self._handles = [safe_open(f, framework="pt", device="cpu") for f in files]
        self._where = {}
        for h in self._handles:
            for k in h.keys():
                self._where.setdefault(k, h)

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def get(self, name: str) -> torch.Tensor:
        if name not in self._where:
            raise KeyError(f"checkpoint has no tensor {name}")
        return self._where[name].get_tensor(name)

    def metadata(self) -> dict:
        return self._handles[0].metadata() or {}


def _is_moe(shape) -> bool:
    return hasattr(shape, "experts")


def hf_projection_name(b: int, name: str) -> str:
    """HF parameter name of projection ``name`` of block ``b``."""
    part = "self_attn" if name in _ATTN else "mlp"
    return f"model.layers.{b}.{part}.{name}.weight"


def hf_experts(ckpt: HFCheckpoint, b: int, shape) -> tuple[torch.Tensor, torch.Tensor,
                                                             torch.Tensor]:
    """(router [E, H], gate_up [E, 2I, H], down [E, H, I]) of MoE block ``b``, from
    the fused layout of transformers 5 (``mlp.experts.gate_up_proj``) or the
    per-expert w1 (gate) / w3 (up) / w2 (down) layout of earlier versions."""
    p = f"model.layers.{b}"
    if f"{p}.mlp.experts.gate_up_proj" in ckpt:
        return (ckpt.get(f"{p}.mlp.gate.weight"), ckpt.get(f"{p}.mlp.experts.gate_up_proj"),
                ckpt.get(f"{p}.mlp.experts.down_proj"))
    q = f"{p}.block_sparse_moe"
    gu = torch.stack([torch.cat([ckpt.get(f"{q}.experts.{e}.w1.weight"),
                                 ckpt.get(f"{q}.experts.{e}.w3.weight")], dim=0)
                      for e in range(shape.experts)])
    dn = torch.stack([ckpt.get(f"{q}.experts.{e}.w2.weight") for e in range(shape.experts)])
    return ckpt.get(f"{q}.gate.weight"), gu, dn


@torch.no_grad()
def pack_block_from_hf(ws, b: int, ckpt: HFCheckpoint, block_projections: tuple[str, ...],
                       device, keep: tuple[str, ...] = ()) -> dict[str, torch.Tensor]:
    """Quantises block ``b``'s projections into its segment (and, for MoE, its
    experts and router). Returns the bf16 device weights of the projections
    named in ``keep`` (selective full fine-tuning needs the true weights)."""
    dev = torch.device(device)
    kept = {}
    tensors = {}
    for name in block_projections:
        w = ckpt.get(hf_projection_name(b, name)).to(dev, torch.bfloat16)
        if name in keep:
            kept[name] = w
        wq, sw = ops.quantize_weight(w)
        tensors[name + ".wq"] = wq
        tensors[name + ".sw"] = sw
    for norm in ("input_layernorm", "post_attention_layernorm"):
        tensors[norm] = ckpt.get(f"model.layers.{b}.{norm}.weight").to(dev, torch.bfloat16)
    ws.pack_block(b, tensors, commit=False)
    if _is_moe(ws.shape):
        router, gu, dn = hf_experts(ckpt, b, ws.shape)
        buf = ws.staging(b)
        for e in range(ws.shape.experts):
            for name, w in (("gate_up", gu[e]), ("down", dn[e])):
                wq, sw = ops.quantize_weight(w.to(dev, torch.bfloat16))
                ws._view(buf, f"experts.{name}.wq")[e].copy_(wq)
                ws._view(buf, f"experts.{name}.sw")[e].copy_(sw)
        ws._view(buf, "router").copy_(router.to(dev, torch.bfloat16))
    ws.commit(b)
    return kept


def _layout_json(ws) -> str:
    return json.dumps({name: [seg.offset, seg.nbytes, list(seg.shape), str(seg.dtype)]
                       for name, seg in ws.layout.items()}, sort_keys=True)


def _shape_json(shape) -> str:
    return json.dumps({"arch": "mixtral" if _is_moe(shape) else "llama",
                       **dataclasses.asdict(shape)}, sort_keys=True)


def save_segments(path: str, ws, embed: torch.Tensor, norm: torch.Tensor,
                  lm_head: torch.Tensor) -> None:
    """Writes every block's packed segment and the resident embedding / head."""
    from safetensors.torch import save_file
    if ws.sharded:
        raise ValueError("a sharded stream holds only its chunk of each segment: save from an "
                         "unsharded one")
    meta = {"format": SEGMENT_FORMAT, "shape": _shape_json(ws.shape),
            "layout": _layout_json(ws), "segment_bytes": str(ws.seg_bytes)}
    save_file({"segments": ws.ram[:, :ws.seg_bytes],
               "model.embed_tokens.weight": embed.detach().cpu().contiguous(),
               "model.norm.weight": norm.detach().cpu().contiguous(),
               "lm_head.weight": lm_head.detach().cpu().contiguous()}, path, metadata=meta)


def is_segment_file(path: str) -> bool:
    if not (os.path.isfile(path) and path.endswith(".safetensors")):
        return False
    try:
        return HFCheckpoint(path).metadata().get("format") == SEGMENT_FORMAT
    except Exception:
        return False


@torch.no_grad()
def load_segments(path: str, ws) -> HFCheckpoint:
    """Copies the saved segments into ``ws`` (this rank's chunk when sharded) after
    checking that the model shape and the segment layout match. Returns the
    opened file (its embedding / head tensors are read by the caller)."""
    from safetensors import safe_open
    ck = HFCheckpoint(path)
    meta = ck.metadata()
    if meta.get("format") != SEGMENT_FORMAT:
        raise ValueError(f"{path} is not a {SEGMENT_FORMAT} file")
    if json.loads(meta["shape"]) != json.loads(_shape_json(ws.shape)):
        raise ValueError(f"{path} holds a model of shape {meta['shape']}, not "
                         f"{_shape_json(ws.shape)}")
    if meta["layout"] != _layout_json(ws):
        raise ValueError(f"{path} was written with a different segment layout")
    with safe_open(path, framework="pt", device="cpu") as f:
        seg = f.get_slice("segments")
        c0 = ws.rank * ws.chunk
        c1 = min(c0 + ws.chunk, ws.seg_bytes)
        for b in range(ws.num_blocks):
            if c1 > c0:
                ws.ram[b, :c1 - c0].copy_(seg[b:b + 1, c0:c1].reshape(-1))
    return ck
