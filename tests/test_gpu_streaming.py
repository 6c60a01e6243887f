"""Expert streaming (ExpertCache.swift:9-102): a .qpack model opened with an
HBM budget below its expert set keeps a bounded slot pool filled from the
layer files on a miss. As MetalModelTests.swift:49-77 does with a small
cacheBudgetGB, the streamed model must give the same logits as the fully
resident one, and the pool counters must show misses beyond the slot count
(evictions) with the slot count bounded."""
import os

import numpy as np
import pytest

import swiftlet_b200 as swl
from conftest import REF_FIXTURES
from swiftlet_b200 import formats

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def container(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("stream") / "tiny-q4.qpack")
    formats.repack(os.path.join(REF_FIXTURES, "tiny-model-q4"), out)
    return out


def test_streamed_pool_matches_resident_pool(container):
    full = swl.QwenCUDAModel(container)
    stride = full.expert_cache.stride
    total = full.config.num_hidden_layers * full.config.num_experts
    budget = 20 * stride / 2**30  # 20 slots of 64 blobs
    small = swl.QwenCUDAModel(container, cache_budget_gb=budget)
    st_f, st_s = swl.DecodeState(64), swl.DecodeState(64)
    prompt = [1, 5, 9, 42, 7, 99, 3, 17, 64, 2]
    # the resident model prefills through the batched kernels, the streaming
    # one token by token (its routing goes to the host layer by layer): the
    # logits agree to f32 reassociation, the greedy tokens exactly
    a = full.step(prompt, st_f)
    b = small.step(prompt, st_s)
    assert np.abs(a - b).max() < 1e-4
    for _ in range(12):
        t = int(np.argmax(a))
        assert t == int(np.argmax(b))
        a = full.step([t], st_f)
        b = small.step([t], st_s)
        assert np.abs(a - b).max() < 1e-4
    s = small.expert_cache
    assert s.slot_count == 20 and s.allocated_slots <= 20
    assert s.misses > 20 and s.hits > 0          # evictions happened, some picks hit
    assert s.hits + s.misses == 22 * 8 * small.config.num_experts_per_tok
    # shrinkCache (QwenMetalModel.swift:324): a smaller, empty pool; the
    # sequence continues with the same logits
    small.shrink_cache(16 * stride / 2**30)
    assert small.expert_cache.slot_count == 16
    t = int(np.argmax(a))
    assert np.abs(full.step([t], st_f) - small.step([t], st_s)).max() < 1e-4
    assert total > 20
