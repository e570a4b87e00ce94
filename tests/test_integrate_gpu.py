"""The reference's own code behind ``backend="cpp"`` on the B200 path
(lema_b200.integrate), against the same reference code on the CPU with the
oracle's W8A8 linears.

1. Llama and Mistral (GQA, 2 kv heads, sliding window longer than the
   sequence): the reference's ``LemaModel(backend="cpp")`` on a 3-block model
   (LoRA r4 on q/v, bf16, eager attention) runs two ``LemaTrainer.train_step``s
   with AdamW on the GPU: weights stream through this library's manager, the
   seven projections of every block are W8A8 (quantised from the streamed
   flat buffer), the boundary activations go to pinned host memory and back.
   The same reference model on the CPU (``backend="python"``) with every
   projection computing the oracle's W8A8 linear runs the same two steps from
   the same LoRA parameters. The losses agree within two bf16 ulps (measured
   on B200: Llama 6.5625 / 6.46875 against 6.5625 / 6.4375 on the CPU, Mistral
   6.53125 / 6.46875 against 6.5 / 6.4375: at most one ulp apart).
   LFM2 (the reference's ``lfm2_moe`` adapter, dense feed-forward layers) runs
   the same comparison twice: with attention blocks only (LoRA on q/v; W8A8
   q/k/v/out_proj and w1/w2/w3) and with short-convolution blocks only (LoRA
   on in_proj; W8A8 in_proj/out_proj and w1/w2/w3); measured on B200,
   6.625 / 6.53125 against 6.65625 / 6.53125 (attention) and 6.78125 / 6.5625
   against 6.78125 / 6.53125 (convolution). A model that mixes the two
   block types does not train under the reference itself: its adapter's
   module pool hands any pooled decoder layer to the next layer
   (src/lema/adapters/_lfm2.py:88-101), so an attention layer can receive a
   convolution layer's module and weight mapping (NaN losses on the CPU).
   Mixtral (4 experts, top-2, GQA) and LFM2 with MoE layers only: the
   attention's q/k/v/o(ut) are W8A8 and the fused experts run as grouped W8A8
   experts (``lema_grouped_w8a8_gemm``, quantised from the streamed 3-D
   weights), against the oracle's experts on the CPU; measured Mixtral 6.625 /
   6.53125 against 6.59375 / 6.5, LFM2-MoE 6.78125 / 6.6875 against 6.71875 /
   6.6875. Their bar is four ulps: the router's bf16 logits differ in the last
   bit between CPU and GPU GEMMs, which can swap nearly tied experts. (The CPU
   side's own losses move by one ulp between runs: its bf16 reductions are
   multithreaded.)
2. GPT-2: the reference's GPT-2 adapter cannot run a training step under the
   transformers version installed here (its ``forward_layer`` takes ``[0]`` of
   the block's output, which transformers 5 returns as a tensor, not a
   tuple). The test therefore drives the adapter's own
   ``construct_layer_module`` with a streamed flat buffer for two layers,
   checks that c_attn / c_proj / c_fc became W8A8 with their Conv1D weights
   transposed, and runs the HF ``GPT2Block`` forward against a CPU block whose
   Conv1D layers compute the oracle's W8A8 linear of the transposed weight
   plus bias; measured on B200, the outputs are the oracle's bit for bit (the
   bar is 1e-3 relative RMS). (The GPT-2 adapter builds a new module for every layer; the
   Llama test above covers pooled modules, whose weights reach the W8A8
   projections through the mapping entries that quantise.)

The reference package is read from baseline/_ref (installed there from the
reference's sources); without it the tests skip.
"""
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def lema_ref():
    if not (REF / "lema" / "__init__.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import lema
    from lema_b200 import integrate
    integrate.enable()
    yield lema
    integrate.disable()


def bf16_ulp(x: float) -> float:
    return float(np.ldexp(1.0, int(np.frexp(abs(x))[1]) - 8))


def _save(d: Path, sd: dict, cfg: dict) -> str:
    from safetensors.torch import save_file
    d.mkdir(parents=True, exist_ok=True)
    save_file({k: v.to(torch.bfloat16).contiguous() for k, v in sd.items()},
              str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(cfg))
    return str(d)


H, HEADS, INTER, LAYERS, VOCAB, SEQ, BATCH = 256, 4, 512, 3, 512, 64, 2


KV_HEADS = {"llama": HEADS, "mistral": 2}


def _decoder_checkpoint(d: Path, kind: str) -> str:
    """A random HF Llama- or Mistral-layout checkpoint (the two adapters share
    the parameter names; Mistral here with GQA and a sliding window)."""
    kv = KV_HEADS[kind] * (H // HEADS)
    g = torch.Generator().manual_seed(71)
    sd = {"model.embed_tokens.weight": 0.5 * torch.randn(VOCAB, H, generator=g),
          "model.norm.weight": 1.0 + 0.1 * torch.randn(H, generator=g),
          "lm_head.weight": 0.05 * torch.randn(VOCAB, H, generator=g)}
    for i in range(LAYERS):
        p = f"model.layers.{i}"
        sd[f"{p}.input_layernorm.weight"] = 1.0 + 0.1 * torch.randn(H, generator=g)
        sd[f"{p}.post_attention_layernorm.weight"] = 1.0 + 0.1 * torch.randn(H, generator=g)
        for n, (o, k) in {"self_attn.q_proj": (H, H), "self_attn.k_proj": (kv, H),
                          "self_attn.v_proj": (kv, H), "self_attn.o_proj": (H, H),
                          "mlp.gate_proj": (INTER, H), "mlp.up_proj": (INTER, H),
                          "mlp.down_proj": (H, INTER)}.items():
            sd[f"{p}.{n}.weight"] = 0.06 * torch.randn(o, k, generator=g)
    cfg = {"model_type": kind,
           "architectures": ["LlamaForCausalLM" if kind == "llama" else "MistralForCausalLM"],
           "hidden_size": H, "num_attention_heads": HEADS, "num_key_value_heads": KV_HEADS[kind],
           "intermediate_size": INTER, "num_hidden_layers": LAYERS, "vocab_size": VOCAB,
           "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "max_position_embeddings": 512,
           "tie_word_embeddings": False, "hidden_act": "silu", "torch_dtype": "bfloat16",
           "dtype": "bfloat16"}
    if kind == "mistral":
        cfg["sliding_window"] = 4096
    return _save(d, sd, cfg)


def _lfm2_checkpoint(d: Path, layer_type: str, dense: bool = True) -> str:
    """A random HF LFM2-MoE checkpoint whose blocks are all of one type
    ("full_attention" or "conv"), with dense feed-forward layers or all MoE
    (4 experts, top-2)."""
    from transformers import Lfm2MoeConfig
    from transformers.models.lfm2_moe.modeling_lfm2_moe import Lfm2MoeForCausalLM
    cfg = Lfm2MoeConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=INTER,
                        moe_intermediate_size=128, num_hidden_layers=LAYERS,
                        num_attention_heads=HEADS, num_key_value_heads=2, num_experts=4,
                        num_experts_per_tok=2, layer_types=[layer_type] * LAYERS,
                        num_dense_layers=LAYERS if dense else 0, max_position_embeddings=512,
                        tie_word_embeddings=False)
    g = torch.Generator().manual_seed(71)
    sd = {}
    for k, v in Lfm2MoeForCausalLM(cfg).state_dict().items():
        if k.endswith("norm.weight"):
            sd[k] = 1.0 + 0.1 * torch.randn(v.shape, generator=g)
        elif k.endswith("conv.conv.weight"):
            sd[k] = 0.3 * torch.randn(v.shape, generator=g)
        elif "embed_tokens" in k:
            sd[k] = 0.5 * torch.randn(v.shape, generator=g)
        else:
            sd[k] = 0.06 * torch.randn(v.shape, generator=g)
    return _save(d, sd, {**cfg.to_dict(), "torch_dtype": "bfloat16", "dtype": "bfloat16"})


def _mixtral_checkpoint(d: Path) -> str:
    """A random HF Mixtral checkpoint (4 experts, top-2; GQA with 2 kv heads)."""
    from transformers import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralForCausalLM
    cfg = MixtralConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=INTER,
                        num_hidden_layers=LAYERS, num_attention_heads=HEADS,
                        num_key_value_heads=2, num_local_experts=4, num_experts_per_tok=2,
                        max_position_embeddings=512, tie_word_embeddings=False,
                        sliding_window=None)
    g = torch.Generator().manual_seed(71)
    sd = {}
    for k, v in MixtralForCausalLM(cfg).state_dict().items():
        if k.endswith("norm.weight"):
            sd[k] = 1.0 + 0.1 * torch.randn(v.shape, generator=g)
        elif "embed_tokens" in k:
            sd[k] = 0.5 * torch.randn(v.shape, generator=g)
        else:
            sd[k] = 0.06 * torch.randn(v.shape, generator=g)
    return _save(d, sd, {**cfg.to_dict(), "torch_dtype": "bfloat16", "dtype": "bfloat16"})


# kind -> (model_type, checkpoint builder, LoRA targets, loss bar in bf16 ulps). The
# MoE models' bar is wider: their router logits come from bf16 GEMMs that differ between
# the CPU and the GPU in the last bit, which can swap the top-k choice of a token whose
# experts are nearly tied (measured: 2 ulps on LFM2-MoE's first step, 1 on Mixtral's).
DECODERS = {
    "llama": ("llama", lambda d: _decoder_checkpoint(d, "llama"), ("q_proj", "v_proj"), 2),
    "mistral": ("mistral", lambda d: _decoder_checkpoint(d, "mistral"), ("q_proj", "v_proj"),
                2),
    "lfm2_attention": ("lfm2_moe", lambda d: _lfm2_checkpoint(d, "full_attention"),
                       ("q_proj", "v_proj"), 2),
    "lfm2_conv": ("lfm2_moe", lambda d: _lfm2_checkpoint(d, "conv"), ("in_proj",), 2),
    "mixtral": ("mixtral", _mixtral_checkpoint, ("q_proj", "v_proj"), 4),
    "lfm2_moe": ("lfm2_moe", lambda d: _lfm2_checkpoint(d, "full_attention", dense=False),
                 ("q_proj", "v_proj"), 4),
}


def _config(lema, path, model_type, device, backend, targets):
    return lema.LemaConfig(model_name_or_path=path, model_type=model_type,
                           gbi_path=os.path.join(path, "model.safetensors"), device=device,
                           dtype="bfloat16", lora_rank=4, lora_alpha=8,
                           lora_target_modules=list(targets), save_steps=0, backend=backend,
                           attn_implementation="eager", max_ram_gb=4.0, max_vram_gb=8.0,
                           vram_fraction=1.0)


def _route_through_oracle(adapter, blocks):
    """CPU model: every projection of a block module the adapter constructs
    computes the oracle's W8A8 linear of the weight it holds at call time, and
    fused MoE experts the oracle's W8A8 experts of theirs."""
    from oracle.torch_ref import OracleExperts, OracleW8A8Linear
    construct = adapter.construct_layer_module
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
             "out_proj", "in_proj", "w1", "w2", "w3")

    def construct_layer_module(layer_id, *a, **k):
        module = construct(layer_id, *a, **k)
        if layer_id in blocks:
            for parent in list(module.modules()):
                for name, child in list(parent.named_children()):
                    if (name == "experts" and hasattr(child, "gate_up_proj")
                            and not getattr(child, "_oracle", False)):
                        child._oracle = True
                        child.forward = (lambda x, i, w, ex=child: OracleExperts(
                            ex.gate_up_proj.detach(), ex.down_proj.detach())(x, i, w))
                        continue
                    if name not in names:
                        continue
                    lin = child.base_layer if hasattr(child, "base_layer") else child
                    if isinstance(lin, torch.nn.Linear) and not getattr(lin, "_oracle", False):
                        lin._oracle = True
                        lin.forward = (lambda x, lin=lin: OracleW8A8Linear.from_linear(lin)(x))
        return module
    adapter.construct_layer_module = construct_layer_module


@pytest.mark.parametrize("kind", list(DECODERS))
def test_reference_decoder_model_trains_through_backend_cpp(lema_ref, cuda_device, tmp_path,
                                                            kind):
    from lema_b200 import _native as N
    from lema_b200._csrc._lema_cpp import LemaMemoryManager
    from lema_b200.modules import W8A8Linear
    from lema_b200.moe import W8A8Experts
    lema = lema_ref
    model_type, build, targets, ulps = DECODERS[kind]
    if model_type == "lfm2_moe":
        pytest.importorskip("transformers.models.lfm2_moe")
    path = build(tmp_path / kind)
    ids = torch.randint(0, VOCAB, (BATCH, SEQ), generator=torch.Generator().manual_seed(5))

    cpu = lema.LemaModel(_config(lema, path, model_type, "cpu", "python", targets))
    blocks = {m["id"] for m in cpu.adapter.get_layer_metadata() if m["type"] == "block"}
    _route_through_oracle(cpu.adapter, blocks)
    cpu.initialize_lora()
    gpu = lema.LemaModel(_config(lema, path, model_type, "cuda", "cpp", targets))
    gpu.initialize_lora()
    assert sorted(gpu.lora_manager.params) == sorted(cpu.lora_manager.params)
    with torch.no_grad():
        for key, p in cpu.lora_manager.params.items():
            for ab in ("A", "B"):
                gpu.lora_manager.params[key][ab].copy_(p[ab].to(cuda_device))

    launches0 = N.kernel_launches
    losses = {}
    for name, model, dev in (("cpu", cpu, "cpu"), ("gpu", gpu, cuda_device)):
        opt = torch.optim.AdamW(model.lora_manager.get_trainable_parameters(), lr=1e-2)
        trainer = model.get_trainer(opt)
        x = ids.to(dev)
        losses[name] = [trainer.train_step(x, labels=x)[1] for _ in range(2)]
        if name == "gpu":
            torch.cuda.synchronize()
            off = trainer.boundary_offload
            assert isinstance(trainer.memory.cpp_mgr, LemaMemoryManager)
            assert off.bytes_out > 0 and off.bytes_in == off.bytes_out, (off.bytes_out,
                                                                          off.bytes_in)
            pool = [m for m in gpu.adapter.module_pool
                    for sub in m.modules() if isinstance(sub, W8A8Linear)]
            assert pool, "no W8A8 projection in the adapter's module pool"
            if kind in ("mixtral", "lfm2_moe"):
                assert any(isinstance(sub, W8A8Experts) for m in gpu.adapter.module_pool
                           for sub in m.modules()), "experts not W8A8"
        trainer.close()
    print(f"[integrate] {kind} losses cpu {losses['cpu']} gpu {losses['gpu']}")
    assert N.kernel_launches > launches0
    for a, b in zip(losses["gpu"], losses["cpu"]):
        assert abs(a - b) <= ulps * bf16_ulp(b), (losses["gpu"], losses["cpu"])


def _gpt2_checkpoint(d: Path):
    from transformers import GPT2Config, GPT2LMHeadModel
    # no dropout: the modules run in training mode, and both sides must be deterministic
    cfg = GPT2Config(n_embd=256, n_layer=2, n_head=4, vocab_size=512, n_positions=128,
                     dtype="bfloat16", attn_implementation="eager", resid_pdrop=0.0,
                     embd_pdrop=0.0, attn_pdrop=0.0)
    torch.manual_seed(0)
    m = GPT2LMHeadModel(cfg)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith(".bias"):
                p.normal_(0.0, 0.1)
    sd = {k: v.clone() for k, v in m.state_dict().items()
          if not k.endswith(".attn.bias") and "masked_bias" not in k}
    return _save(d, sd, {**cfg.to_dict(), "torch_dtype": "bfloat16"}), sd, cfg


def test_reference_gpt2_adapter_binds_conv1d_as_w8a8(lema_ref, cuda_device, tmp_path):
    from transformers.models.gpt2.modeling_gpt2 import GPT2Block

    from lema_b200.modules import W8A8Linear
    from oracle.torch_ref import OracleW8A8Linear
    lema = lema_ref
    dev = cuda_device
    path, sd, hf_cfg = _gpt2_checkpoint(tmp_path / "gpt2")
    model = lema.LemaModel(_config(lema, path, "gpt2", "cuda", "cpp", ("c_attn",)))
    model.initialize_lora()
    adapter = model.adapter
    g = torch.Generator().manual_seed(3)
    with torch.no_grad():  # B non-zero so the LoRA branch contributes
        for p in model.lora_manager.params.values():
            p["B"].copy_((0.05 * torch.randn(p["B"].shape, generator=g)).to(p["B"]))
    x = (0.5 * torch.randn(2, 48, hf_cfg.n_embd, generator=g)).to(torch.bfloat16)
    for layer_id in (1, 2):
        names = adapter.get_param_names_for_layer(layer_id)
        flat = torch.cat([sd[n].reshape(-1).to(torch.bfloat16) for n in names]).to(dev)
        module = adapter.construct_layer_module(layer_id, flat, model.lora_manager)
        for part in (module.attn.c_attn, module.attn.c_proj, module.mlp.c_fc,
                     module.mlp.c_proj):
            base = part.base_layer if hasattr(part, "base_layer") else part
            assert isinstance(base, W8A8Linear), type(base)
        with torch.no_grad():
            y = module(x.to(dev))
            y = y[0] if isinstance(y, tuple) else y
        # CPU: the HF block with the same weights, Conv1D layers on the oracle
        ref = GPT2Block(hf_cfg).to(torch.bfloat16)
        prefix = f"transformer.h.{layer_id - 1}."
        ref.load_state_dict({k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)},
                            strict=False)
        for parent, name in ((ref.attn, "c_attn"), (ref.attn, "c_proj"), (ref.mlp, "c_fc"),
                             (ref.mlp, "c_proj")):
            conv = getattr(parent, name)
            setattr(parent, name, OracleW8A8Linear(conv.weight.t(), conv.bias))
        lora = model.lora_manager.params[f"{layer_id}.attn.c_attn"] \
            if f"{layer_id}.attn.c_attn" in model.lora_manager.params else None
        if lora is not None:
            base = ref.attn.c_attn
            a, b = lora["A"].detach().cpu(), lora["B"].detach().cpu()

            class _Lora(torch.nn.Module):
                def forward(self, t):
                    return base(t) + (t @ a.t() @ b.t()) * (8 / 4)
            ref.attn.c_attn = _Lora()
        with torch.no_grad():
            yr = ref(x)
            yr = yr[0] if isinstance(yr, tuple) else yr
        err = (y.float().cpu() - yr.float())
        rel = err.pow(2).mean().sqrt().item() / yr.float().pow(2).mean().sqrt().item()
        print(f"[integrate] gpt2 layer {layer_id}: rel-rms {rel:.3e}")
        assert rel <= 1e-3, rel  # measured 0: the same bits as the oracle block
        adapter.release_layer_module(module)
