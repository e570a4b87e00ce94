"""CPU tests of how a device-side failure reaches the host: the pinned error
word that ``lema_device_error_async`` fills is checked before every training
step, and a nonzero word raises LemaError from the trainer instead of letting
training go on with a wrong tile."""
import pytest
import torch

from lema_b200 import _native as N
from lema_b200.trainer import StreamedLoraTrainer


def test_watch_raises_on_a_nonzero_word_and_clears_it():
    host = torch.zeros(1, dtype=torch.int32)
    watch = N.DeviceErrorWatch(host=host)
    watch.check()  # zero: nothing raised
    host[0] = 0x104
    with pytest.raises(N.LemaError) as e:
        watch.check()
    assert e.value.code == N.LEMA_ERR_DEVICE
    assert "0x104" in str(e.value) and "partial accumulators" in str(e.value)
    watch.check()  # the word was cleared by the raise


def test_trainer_step_raises_before_running_when_the_word_is_set():
    tr = StreamedLoraTrainer.__new__(StreamedLoraTrainer)  # no GPU: only the check runs
    tr.errors = N.DeviceErrorWatch(host=torch.tensor([0x102], dtype=torch.int32))
    with pytest.raises(N.LemaError) as e:
        tr.train_step(torch.zeros(1, 4, dtype=torch.int64))
    assert e.value.code == N.LEMA_ERR_DEVICE and "0x102" in str(e.value)
    tr.errors.host[0] = 0x103
    with pytest.raises(N.LemaError):
        tr.check_device_errors()


def test_async_error_entry_rejects_a_null_word():
    lib = N.lib()
    assert lib.lema_device_error_async(None, None) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_gemm_set_test_hooks(0, -1) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_gemm_set_test_hooks(0, 0) == N.LEMA_OK  # defaults; clears the message
    assert N.last_error() == ""
