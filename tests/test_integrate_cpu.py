"""CPU tests of lema_b200.integrate: the reference's backend="cpp" import
resolves to this library's manager, enable()/disable() wrap and restore the
reference's LemaModel, a mapping entry of a W8A8 projection quantises the
flat-buffer view it is given (transposed for GPT-2's Conv1D), and the
projections listed for LFM2 are linears the reference adapter streams."""
import sys
from pathlib import Path

import pytest
import torch

from lema_b200 import integrate

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture
def lema_ref():
    if not (REF / "lema" / "__init__.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import lema
    return lema


def test_backend_cpp_imports_this_librarys_manager(lema_ref):
    import lema._tensorstore as ts

    from lema_b200._csrc import _lema_cpp
    integrate.install_backend()
    assert ts.HAS_CPP_BACKEND and ts._lema_cpp is _lema_cpp
    assert sys.modules["lema._csrc._lema_cpp"] is _lema_cpp
    # the four manager calls the reference's transfer engine makes
    # (src/lema/_tensorstore.py:123, 154, 280, 297)
    for name in ("register_vram_slot", "register_ram_buffer", "async_transfer_to_vram",
                 "wait_vram_transfer"):
        assert callable(getattr(_lema_cpp.LemaMemoryManager, name))


def test_enable_wraps_and_disable_restores_the_model_class(lema_ref):
    cls = lema_ref.LemaModel
    init, get_trainer = cls.__init__, cls.get_trainer
    integrate.enable()
    try:
        assert cls.__init__ is not init and cls.get_trainer is not get_trainer
        integrate.enable()  # idempotent
    finally:
        integrate.disable()
    assert cls.__init__ is init and cls.get_trainer is get_trainer


class _Recorder:
    def __init__(self):
        self.got = None

    def requantize_(self, w):
        self.got = w


def test_mapping_entry_quantises_the_view_it_is_given():
    rec = _Recorder()
    slot = integrate._QuantizingSlot(rec, transpose=False)
    flat = torch.arange(24, dtype=torch.float32)
    view = flat[4:16].view(3, 4)
    assert slot.data is slot
    slot.data.copy_(view, non_blocking=True)  # what the reference's binding loop calls
    assert rec.got.data_ptr() == view.data_ptr() and tuple(rec.got.shape) == (3, 4)
    conv = integrate._QuantizingSlot(rec, transpose=True)
    conv.data.copy_(view)
    assert tuple(rec.got.shape) == (4, 3) and torch.equal(rec.got, view.t())


def test_offload_eligibility_rules():
    off = integrate.BoundaryOffload.__new__(integrate.BoundaryOffload)
    x = torch.randn(2, 8)
    assert not off._eligible(x)  # CPU tensors stay where they are
    assert not off._eligible(torch.zeros(2, 3, dtype=torch.int64))


def test_lfm2_projections_are_streamed_linears(lema_ref):
    """Every name listed for the reference's LFM2 adapter is an nn.Linear of its
    convolution and attention blocks, and its weight is one of the parameters
    the adapter streams for that layer (src/lema/adapters/_lfm2.py:48-75), so
    the mapping has an entry to quantise."""
    pytest.importorskip("transformers.models.lfm2_moe")
    from transformers import Lfm2MoeConfig

    from lema.adapters import get_adapter
    cfg = Lfm2MoeConfig(vocab_size=64, hidden_size=32, intermediate_size=64,
                        moe_intermediate_size=32, num_hidden_layers=2, num_attention_heads=4,
                        num_key_value_heads=2, num_experts=4, num_experts_per_tok=2,
                        layer_types=["conv", "full_attention"], num_dense_layers=2,
                        max_position_embeddings=16)
    adapter = get_adapter("lfm2_moe", cfg.to_dict())
    names = integrate.PROJECTIONS[type(adapter).__name__]
    seen = set()
    for layer_id in (1, 2):
        module = adapter.construct_layer_module(layer_id)
        streamed = set(adapter.get_param_names_for_layer(layer_id))
        prefix = f"model.layers.{layer_id - 1}."
        for full, child in module.named_modules():
            if full.rsplit(".", 1)[-1] in names:
                assert isinstance(child, torch.nn.Linear), (full, type(child))
                assert prefix + full + ".weight" in streamed, full
                seen.add(full.rsplit(".", 1)[-1])
    assert seen == set(names)


def test_fused_experts_are_recognised_and_their_parts_dispatched():
    """HF's fused-experts modules (Mixtral, LFM2-MoE) are the ones the W8A8
    conversion takes; a dense MLP is not; each streamed 3-D parameter's mapping
    entry re-quantises its own half of the W8A8 experts."""
    from transformers import LlamaConfig, MixtralConfig
    from transformers.models.llama.modeling_llama import LlamaMLP
    from transformers.models.mixtral.modeling_mixtral import MixtralExperts
    cfg = MixtralConfig(hidden_size=32, intermediate_size=64, num_local_experts=4,
                        num_experts_per_tok=2, num_attention_heads=4, num_key_value_heads=2)
    assert integrate._is_fused_experts(MixtralExperts(cfg))
    assert not integrate._is_fused_experts(
        LlamaMLP(LlamaConfig(hidden_size=32, intermediate_size=64)))
    try:
        from transformers import Lfm2MoeConfig
        from transformers.models.lfm2_moe.modeling_lfm2_moe import Lfm2MoeExperts
        lcfg = Lfm2MoeConfig(hidden_size=32, moe_intermediate_size=16, num_experts=4)
        assert integrate._is_fused_experts(Lfm2MoeExperts(lcfg))
    except ImportError:
        pass

    class _Experts:
        def __init__(self):
            self.got = []

        def requantize_gate_up_(self, w):
            self.got.append(("gate_up", tuple(w.shape)))

        def requantize_down_(self, w):
            self.got.append(("down", tuple(w.shape)))

    ex = _Experts()
    flat = torch.zeros(4 * 8 * 4 + 4 * 4 * 4)
    gu = integrate._QuantizingSlot(integrate._ExpertsPart(ex, "gate_up_proj"), False)
    dn = integrate._QuantizingSlot(integrate._ExpertsPart(ex, "down_proj"), False)
    gu.data.copy_(flat[:128].view(4, 8, 4))
    dn.data.copy_(flat[128:].view(4, 4, 4))
    assert ex.got == [("gate_up", (4, 8, 4)), ("down", (4, 4, 4))]


def test_every_reference_adapter_has_a_projection_list(lema_ref):
    """Each adapter the reference registers (src/lema/adapters/__init__.py) has its
    W8A8 projection list here, so ``backend="cpp"`` never meets an adapter it
    cannot convert."""
    from lema.adapters import _ADAPTER_REGISTRY
    missing = [cls.__name__ for cls in _ADAPTER_REGISTRY.values()
               if cls.__name__ not in integrate.PROJECTIONS]
    assert not missing, missing
