"""GPU: a device-side bounded wait that runs out is reported, and the next call is correct.

The test hook ``uocr_moe_test_wait_extra(1)`` makes the decode down phase wait, per slot, for one
gate/up arrival that never comes, so the bounded waits give up after their budget (a counter that
nothing completes: no fault, no trap, the context stays usable). The call must then write NaN over
its output (never stale values); until the status is read, later calls write NaN too; the status
read must return UOCR_EDEVICE once and clear it, and the next call, with the hook off, must give
the same bits as before the failure.
"""

from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture
def hook(uocr):
    lib = uocr.load()
    yield lib
    assert lib.uocr_moe_test_wait_extra(0) == 0


@pytest.mark.parametrize("int8", [False, True])
def test_expired_wait_is_reported_and_the_next_call_is_correct(uocr, hook, int8):
    lib = hook
    UocrError = importlib.import_module("unlimited-ocr-max_b200._lib").UocrError
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    cfg = uocr.MoEConfig(int8_experts=int8)
    moe = uocr.UocrMoE(cfg, device=DEV).load_state_dict(synth.layer_state(cfg, 61, device=DEV))
    x = synth.hidden_states(8, 1280, 62, device=DEV)
    good = moe.decode_rows(x, check_status=True).clone()
    assert torch.isfinite(good).all()

    assert lib.uocr_moe_test_wait_extra(1) == 0
    bad = moe.decode_rows(x)
    assert lib.uocr_moe_test_wait_extra(0) == 0
    torch.cuda.synchronize()
    assert torch.isnan(bad).all()  # the failed call wrote NaN, not a stale or partial result
    with pytest.raises(UocrError) as e:
        moe.check_status()
    assert e.value.code == 3 and "bounded wait" in str(e.value)
    moe.check_status()  # read once: cleared

    again = moe.decode_rows(x, check_status=True)
    assert torch.equal(again, good)
    # with the failure left unread, later calls write NaN (their counters are not trusted) ...
    assert lib.uocr_moe_test_wait_extra(1) == 0
    moe.decode_rows(x)
    assert lib.uocr_moe_test_wait_extra(0) == 0
    assert torch.isnan(moe.decode_rows(x)).all()
    with pytest.raises(UocrError):
        moe.check_status()
    # ... and once it is read, the layer computes the same bits again, batch after batch
    assert torch.equal(moe.decode_rows(x, check_status=True), good)
    for _ in range(5):
        assert torch.equal(moe.decode_rows(x), good)
    moe.check_status()
