"""The allocation-free expert SwiGLU entry point (for callers that cannot call
cudaMalloc, e.g. a host runtime that owns all device memory in its own arena)
gives the same result as the allocating kernel-level entry point and as the
CPU oracle, on two calls in a row that share its library-wide scratch array,
up to the scratch's size limit, and reports no timed-out wait.

Collected last on purpose (file name), so a run that stops at the first
failure has already run every other test."""
import numpy as np
import pytest

import oracle
import swiftlet_b200 as swl

pytestmark = pytest.mark.gpu


def _bf16(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _matrix(rng, rows, cols, group, bits):
    packed = rng.integers(0, 2**32, size=rows * cols * bits // 32, dtype=np.uint64).astype(np.uint32)
    scales = _bf16(np.abs(rng.normal(0, 0.01, rows * cols // group)))
    biases = _bf16(rng.normal(0, 0.01, rows * cols // group))
    return packed, scales, biases


def _device(torch, mat, rows, cols, group, bits):
    t = [torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)).cuda() for a in mat]
    m = swl.swl_affine_matrix(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), rows, cols, bits, group, 1)
    return m, t


def _run(torch, mats, hidden, inter, group, bits, rng, calls=2):
    """Two calls in a row (the second reuses the scratch the first left):
    each against the allocating entry point and the CPU oracle."""
    gate, up, down = mats
    keep = []
    dg, t = _device(torch, gate, inter, hidden, group, bits); keep += t
    du, t = _device(torch, up, inter, hidden, group, bits); keep += t
    dd, t = _device(torch, down, hidden, inter, group, bits); keep += t
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(calls):
        x = rng.normal(0, 1, hidden).astype(np.float32)
        ref = swl.expert_swiglu(gate, up, down, hidden, inter, group, bits, x)
        cpu = oracle.expert_swiglu(gate, up, down, hidden, inter, group, bits, x)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((hidden,), float("nan"), dtype=torch.float32, device="cuda")
        swl.expert_swiglu_noalloc(dg, du, dd, dx.data_ptr(), dy.data_ptr(), torch.cuda.current_stream().cuda_stream,
                                  d_status=status.data_ptr())
        torch.cuda.synchronize()
        y = dy.cpu().numpy()
        assert int(status.item()) == 0, "a bounded wait in the expert kernels gave up"
        scale = np.abs(cpu).max() + 1e-6
        # the tolerance of the kernel-level SwiGLU parity tests (test_gpu_kernels.py)
        assert np.abs(y - ref).max() / scale < 1e-5, call
        assert np.abs(y - cpu).max() / scale < 1e-5, call


def test_noalloc_expert_swiglu_matches_allocating_entry_point_and_oracle():
    import torch
    hidden, inter, group, bits = 2048, 512, 64, 4
    rng = np.random.default_rng(77)
    mats = (_matrix(rng, inter, hidden, group, bits), _matrix(rng, inter, hidden, group, bits),
            _matrix(rng, hidden, inter, group, bits))
    _run(torch, mats, hidden, inter, group, bits, rng)


@pytest.mark.parametrize("inter,group", [(16384, 64), (16352, 32)])
def test_noalloc_at_the_scratch_limit(inter, group):
    """The largest intermediate the scratch holds (16384 values), and one that
    is not a multiple of 64; the down projection's input is then too long for
    the tensor-core kernels and takes the register-streaming ones."""
    import torch
    hidden, bits = 256, 4
    rng = np.random.default_rng(inter)
    mats = (_matrix(rng, inter, hidden, group, bits), _matrix(rng, inter, hidden, group, bits),
            _matrix(rng, hidden, inter, group, bits))
    _run(torch, mats, hidden, inter, group, bits, rng)


def test_noalloc_rejects_oversized_intermediate():
    inter = 16384 + 64  # one group past the scratch's 16384 values; rejected before any launch
    gate = swl.swl_affine_matrix(256, 256, 256, inter, 2048, 4, 64, 1)
    down = swl.swl_affine_matrix(256, 256, 256, 2048, inter, 4, 64, 1)
    with pytest.raises(swl.SwiftletError) as err:
        swl.expert_swiglu_noalloc(gate, gate, down, 256, 256)
    assert err.value.code == swl.SWL_ERR_CAPACITY
    assert "16384" in str(err.value)
