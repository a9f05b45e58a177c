"""Partition accounting on the GPU: a model and a session hold exactly the
ledger the host planned before allocating (class by class), a decode step
adds nothing, closing returns every byte, and with a policy limit set the
allocation that would pass it fails as ALLOCATION (src/partition.rs:111-114)
while the limit itself admits an exact fit.
"""

import gc
from dataclasses import astuple, fields

import pytest

pytestmark = pytest.mark.gpu

CTX = 96


def _sms() -> int:
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.fixture
def quiet_gc():
    """No collection of other tests' objects while byte counts are compared."""
    gc.collect()
    gc.disable()
    try:
        yield
    finally:
        gc.enable()


def _delta(a, b):
    from faber_runtime_b200.partition import PartitionLedger
    return PartitionLedger(*(y - x for x, y in zip(astuple(a), astuple(b))))


def _without_module(led):
    return {f.name: getattr(led, f.name) for f in fields(led) if f.name != "module_storage_bytes"}


def test_model_and_session_hold_exactly_the_plan(cuda, quiet_gc):
    from faber_runtime_b200 import TINY, DeviceModel, ForwardRun, synth
    from faber_runtime_b200 import partition as pt
    before = pt.usage(0)
    plan = pt.plan(TINY, CTX, sessions=1, sms=_sms())
    model = DeviceModel(TINY, synth.model_tensors(TINY, 5))
    run = ForwardRun(model, context_length=CTX)
    held = pt.usage(0)
    assert _without_module(_delta(before, held)) == _without_module(plan)
    assert held.module_storage_bytes == plan.module_storage_bytes
    run.push_tokens([1, 2, 3, 4])
    run.position_logits()
    assert pt.usage(0) == held  # decoding allocates nothing further
    run.close()
    model.close()
    assert _without_module(pt.usage(0)) == _without_module(before)


def test_policy_limit_makes_growth_an_allocation_failure(cuda, quiet_gc):
    from faber_runtime_b200 import TINY, DeviceModel, FaberError, ForwardRun, synth
    from faber_runtime_b200 import _lib
    from faber_runtime_b200 import partition as pt
    before = pt.usage(0)
    held = before.total_bytes()
    plan = pt.plan(TINY, CTX, sessions=1, sms=_sms())
    needed = plan.total_bytes() - (plan.module_storage_bytes if before.module_storage_bytes else 0)
    try:
        if held:
            with pytest.raises(FaberError) as e:
                pt.set_limit(0, held - 1)  # below what the device already holds
            assert e.value.code == _lib.BUDGET_EXCEEDED
        # half the weights: the upload stops at the limit and frees what it placed
        pt.set_limit(0, held + plan.weight_bytes // 2)
        with pytest.raises(FaberError) as e:
            DeviceModel(TINY, synth.model_tensors(TINY, 5))
        assert e.value.code == _lib.ALLOCATION
        assert _without_module(pt.usage(0)) == _without_module(before)
        # one byte short: the model fits, the session's last buffer does not
        pt.set_limit(0, held + needed - 1)
        model = DeviceModel(TINY, synth.model_tensors(TINY, 5))
        with pytest.raises(FaberError) as e:
            ForwardRun(model, context_length=CTX)
        assert e.value.code == _lib.ALLOCATION
        model.close()
        assert _without_module(pt.usage(0)) == _without_module(before)
        # an exact fit is admitted
        pt.set_limit(0, held + needed)
        model = DeviceModel(TINY, synth.model_tensors(TINY, 5))
        run = ForwardRun(model, context_length=CTX)
        assert pt.usage(0).total_bytes() == held + needed
        run.push_tokens([7, 8])
        run.close()
        model.close()
    finally:
        pt.set_limit(0, 0)
    assert _without_module(pt.usage(0)) == _without_module(before)
