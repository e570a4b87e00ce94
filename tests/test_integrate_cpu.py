"""CPU tests of lema_b200.integrate: the reference's backend="cpp" import
resolves to this library's manager, enable()/disable() wrap and restore the
reference's LemaModel, and a mapping entry of a W8A8 projection quantises the
flat-buffer view it is given (transposed for GPT-2's Conv1D)."""
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
