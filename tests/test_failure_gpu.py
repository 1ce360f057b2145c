"""Failure detection without faulting a GPU: a device wait that nothing will
satisfy gives up after its time limit and reports an error status that the
host reads, the context stays usable, and an engine step that finds the
error flag set raises instead of returning tokens."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_times_out_with_status_and_context_survives():
    from kunserve_b200.ops import native
    C = native()
    C.error_flag(True)
    H = 512
    h = torch.zeros(2, H, device="cuda", dtype=torch.bfloat16)
    rb = torch.zeros(2 * H, device="cuda", dtype=torch.bfloat16)
    flags = torch.zeros(4, device="cuda", dtype=torch.int32)     # nobody will ever write epoch 7
    t0 = time.time()
    C.tp_reduce(rb.data_ptr(), 1, 2 * H, h, flags.data_ptr(), 7)
    torch.cuda.synchronize()
    waited = time.time() - t0
    err = int(C.error_flag(True))
    assert err & 0xff == 5, err        # peer flag never arrived
    assert 1.0 < waited < 30.0, waited
    # the context is intact: a GEMM right after still computes correctly
    A = torch.randn(64, 256, device="cuda").bfloat16()
    B = torch.randn(512, 256, device="cuda").bfloat16()
    out = torch.empty(64, 512, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, C.EPI_BF16, None, 0, 16)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert ((out.float() - ref).norm() / ref.norm()).item() < 1e-2
    assert int(C.error_flag(True)) == 0


def test_engine_step_raises_on_device_error_then_recovers():
    from kunserve_b200.config import ModelConfig, ParallelConfig
    from kunserve_b200.engine.native_runner import NativeRunner
    from kunserve_b200.engine.step import StepInput
    from kunserve_b200.kv.layout import KVLayout
    from kunserve_b200.ops import native
    C = native()
    mc = ModelConfig("tiny-llama-128", dtype="bf16")
    lay = KVLayout(16, 2, 16, 2, 128, 2)
    run = NativeRunner(mc, ParallelConfig(), lay, torch.device("cuda:0"), max_batch_tokens=256, max_batch_size=8)
    step = StepInput([0], [[1, 2, 3]], [0], [[0]], [1], 0, 2, temperature=[0.0], seeds=[0])
    C.error_flag(True)
    C.raise_error_flag(6, 12345)           # as a failed bounds check would
    with pytest.raises(RuntimeError, match="device error flag"):
        run.step(step)
    C.error_flag(True)
    assert len(run.step(step)) == 1
