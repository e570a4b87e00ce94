"""Host side of checkpoint loading (no GPU): the shard index, the HF parameter
names the reference's adapters request, both Mixtral expert layouts, and the
int8 segment file format (round trip, its shape and layout checks, a sharded
rank's chunk)."""
import types

import pytest
import torch
from safetensors.torch import save_file

from lema_b200 import checkpoint as ckp
from lema_b200.llama import LlamaShape
from lema_b200.tensorstore import _Seg


def test_shard_index_and_names(tmp_path):
    a = {"model.layers.0.self_attn.q_proj.weight": torch.arange(6.).view(2, 3)}
    b = {"model.layers.0.mlp.down_proj.weight": torch.ones(3, 2)}
    save_file(a, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file(b, str(tmp_path / "model-00002-of-00002.safetensors"))
    ck = ckp.HFCheckpoint(str(tmp_path))
    assert ckp.hf_projection_name(0, "q_proj") in ck
    assert ckp.hf_projection_name(0, "down_proj") in ck
    assert ckp.hf_projection_name(0, "up_proj") == "model.layers.0.mlp.up_proj.weight"
    assert torch.equal(ck.get("model.layers.0.self_attn.q_proj.weight"), a[
        "model.layers.0.self_attn.q_proj.weight"])
    with pytest.raises(KeyError):
        ck.get("model.layers.1.self_attn.q_proj.weight")
    with pytest.raises(FileNotFoundError):
        ckp.HFCheckpoint(str(tmp_path / "missing"))


def test_expert_layouts_agree(tmp_path):
    E, H, I = 3, 4, 5
    g = torch.Generator().manual_seed(0)
    w1 = torch.randn(E, I, H, generator=g)
    w3 = torch.randn(E, I, H, generator=g)
    w2 = torch.randn(E, H, I, generator=g)
    router = torch.randn(E, H, generator=g)
    legacy = {"model.layers.1.block_sparse_moe.gate.weight": router}
    for e in range(E):
        legacy[f"model.layers.1.block_sparse_moe.experts.{e}.w1.weight"] = w1[e]
        legacy[f"model.layers.1.block_sparse_moe.experts.{e}.w3.weight"] = w3[e]
        legacy[f"model.layers.1.block_sparse_moe.experts.{e}.w2.weight"] = w2[e]
    fused = {"model.layers.1.mlp.gate.weight": router,
             "model.layers.1.mlp.experts.gate_up_proj": torch.cat([w1, w3], dim=1),
             "model.layers.1.mlp.experts.down_proj": w2}
    save_file(legacy, str(tmp_path / "legacy.safetensors"))
    save_file(fused, str(tmp_path / "fused.safetensors"))
    shape = types.SimpleNamespace(experts=E)
    r0, gu0, dn0 = ckp.hf_experts(ckp.HFCheckpoint(str(tmp_path / "legacy.safetensors")), 1, shape)
    r1, gu1, dn1 = ckp.hf_experts(ckp.HFCheckpoint(str(tmp_path / "fused.safetensors")), 1, shape)
    assert gu0.shape == (E, 2 * I, H) and dn0.shape == (E, H, I)
    for x, y in ((r0, r1), (gu0, gu1), (dn0, dn1)):
        assert torch.equal(x, y)


def _fake_segments(seed, shape, rank=0, world=1):
    layout = {"q_proj.wq": _Seg(0, 64, (8, 8), torch.int8),
              "q_proj.sw": _Seg(128, 32, (8,), torch.float32)}
    seg_bytes = 256
    chunk = seg_bytes // world
    g = torch.Generator().manual_seed(seed)
    ram = torch.randint(0, 256, (3, chunk), generator=g, dtype=torch.int32).to(torch.uint8)
    return types.SimpleNamespace(shape=shape, layout=layout, seg_bytes=seg_bytes, num_blocks=3,
                                 sharded=world > 1, rank=rank, chunk=chunk, ram=ram)


def test_segment_file_round_trip_and_checks(tmp_path):
    shape = LlamaShape(hidden=64, heads=2, kv_heads=2, intermediate=96, vocab=32, layers=3)
    src = _fake_segments(1, shape)
    path = str(tmp_path / "w8a8.safetensors")
    emb, norm, head = torch.randn(32, 64), torch.ones(64), torch.randn(32, 64)
    ckp.save_segments(path, src, emb, norm, head)
    assert ckp.is_segment_file(path)
    dst = _fake_segments(2, shape)
    ck = ckp.load_segments(path, dst)
    assert torch.equal(dst.ram, src.ram)
    assert torch.equal(ck.get("model.embed_tokens.weight"), emb)
    # a sharded rank reads only its chunk
    half = _fake_segments(3, shape, rank=1, world=2)
    ckp.load_segments(path, half)
    assert torch.equal(half.ram, src.ram[:, 128:256])
    # a different model shape or segment layout is refused
    other = _fake_segments(4, LlamaShape(hidden=64, heads=2, kv_heads=2, intermediate=96,
                                         vocab=32, layers=4))
    with pytest.raises(ValueError, match="shape"):
        ckp.load_segments(path, other)
    relaid = _fake_segments(5, shape)
    relaid.layout = dict(relaid.layout, extra=_Seg(192, 16, (16,), torch.uint8))
    with pytest.raises(ValueError, match="layout"):
        ckp.load_segments(path, relaid)
    # a sharded stream cannot save, a plain checkpoint is not a segment file
    with pytest.raises(ValueError):
        ckp.save_segments(str(tmp_path / "x.safetensors"), half, emb, norm, head)
    save_file({"w": torch.ones(2)}, str(tmp_path / "plain.safetensors"))
    assert not ckp.is_segment_file(str(tmp_path / "plain.safetensors"))
    assert not ckp.is_segment_file(str(tmp_path))


def test_corrupted_or_truncated_files_raise(tmp_path):
    """A corrupted safetensors header and a truncated segment file surface as
    Python exceptions (host-side fault injection); neither is taken for a
    segment file."""
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\xff" * 64)
    assert not ckp.is_segment_file(str(bad))
    with pytest.raises(Exception):
        ckp.HFCheckpoint(str(bad))
    shape = LlamaShape(hidden=64, heads=2, kv_heads=2, intermediate=96, vocab=32, layers=3)
    good = str(tmp_path / "w8a8.safetensors")
    ckp.save_segments(good, _fake_segments(1, shape), torch.zeros(32, 64), torch.ones(64),
                      torch.zeros(32, 64))
    data = open(good, "rb").read()
    cut = tmp_path / "cut.safetensors"
    cut.write_bytes(data[: len(data) // 2])
    with pytest.raises(Exception):
        ckp.load_segments(str(cut), _fake_segments(2, shape))
