"""Cache operations on the paged per-stream rings, bit-exact against the CPU model (oracle/cache_ring.py) fed the
same row payloads: append / roll / gather / evict over random permutations of stream ids, k in {1, 2, 7, 14},
5% of streams evicted and refilled per step (the cache microbenchmark's access pattern), plus pool exhaustion
with rollback and page accounting."""

import numpy as np
import pytest
import torch

import ud
from oracle.cache_ring import RingModel

pytestmark = pytest.mark.gpu

NL, D, L = 3, 1024, 70


@pytest.fixture(scope="module", params=[ud.DTYPE_BF16, ud.DTYPE_F32], ids=["bf16", "f32"])
def ceng(request):
    e = ud.Engine(ud.default_config(n_layers=NL, sub_channels=0, joint_dim=0, max_streams=24, max_batch=24,
                                    max_chunk_frames=14, dtype=request.param))
    yield e
    e.close()


def _payload(shape, dtype_code, gen):
    """Random bit patterns in the engine's element width, as a cuda tensor and its numpy twin."""
    if dtype_code == ud.DTYPE_BF16:
        t = torch.randint(-32768, 32768, shape, generator=gen, dtype=torch.int32).to(torch.int16)
        return t.cuda(), t.numpy().view(np.uint16)
    t = torch.randint(-2**31, 2**31 - 1, shape, generator=gen, dtype=torch.int32)
    return t.cuda(), t.numpy().view(np.float32)


def test_append_roll_gather_evict_bit_exact(ceng):
    e = ceng
    npdt = np.uint16 if e.cfg.dtype == ud.DTYPE_BF16 else np.float32
    tdt = torch.int16 if e.cfg.dtype == ud.DTYPE_BF16 else torch.int32
    model = RingModel(NL, D, L, 8, npdt)
    ids = [e.open(0) for _ in range(24)]
    for s in ids:
        model.open(s)
    free0, total, _ = e.pool_info()
    rng = np.random.default_rng(0)
    gen = torch.Generator().manual_seed(0)
    for step in range(30):
        k = int(rng.choice([1, 2, 7, 14]))
        batch = [int(s) for s in rng.permutation(ids)[: int(rng.integers(1, len(ids) + 1))]]
        kv_t, kv_np = _payload((len(batch), NL, 2, k, D), e.cfg.dtype, gen)
        cv_t, cv_np = _payload((len(batch), NL, k, D), e.cfg.dtype, gen)
        torch.cuda.synchronize()
        e.cache_append(batch, k, kv_t.data_ptr(), cv_t.data_ptr())
        e.cache_roll(batch, k)
        for i, s in enumerate(batch):
            model.append(s, kv_np[i], cv_np[i])
            model.roll(s, k)
        order = [int(s) for s in rng.permutation(ids)]
        g_kv = torch.empty((len(order), NL, 2, L, D), dtype=tdt, device="cuda")
        g_cv = torch.empty((len(order), NL, 8, D), dtype=tdt, device="cuda")
        e.cache_gather(order, g_kv.data_ptr(), g_cv.data_ptr())
        e.synchronize()
        got_kv = g_kv.cpu().numpy().view(npdt)
        got_cv = g_cv.cpu().numpy().view(npdt)
        for i, s in enumerate(order):
            ref_kv, ref_cv = model.gather(s)
            assert np.array_equal(got_kv[i].view(np.uint8), ref_kv.view(np.uint8)), (step, s)
            assert np.array_equal(got_cv[i].view(np.uint8), ref_cv.view(np.uint8)), (step, s)
            cl, head, _ = e.info(s)
            assert (cl, head) == model.info(s)
        # 5% evicted and refilled (fresh zero caches, same ids)
        ev = [int(s) for s in rng.choice(ids, size=max(1, len(ids) // 20), replace=False)]
        e.cache_evict(ev)
        for s in ev:
            model.evict(s)
        # a stream never holds more than the pages its window needs
        used = total - e.pool_info()[0]
        assert used <= sum((model.info(s)[0] + 15) // 16 + 1 for s in ids)
    for s in ids:
        e.close_stream(s)
    assert e.pool_info()[0] == free0


def test_pool_exhaustion_rolls_back(ceng):
    e = ud.Engine(ud.default_config(n_layers=1, sub_channels=0, joint_dim=0, max_streams=4, max_batch=4,
                                    max_chunk_frames=14, n_pages=3, dtype=ceng.cfg.dtype))
    try:
        a, b, c, d = (e.open(0) for _ in range(4))
        tdt = torch.int16 if e.cfg.dtype == ud.DTYPE_BF16 else torch.int32
        kv = torch.zeros((4, 1, 2, 14, D), dtype=tdt, device="cuda")
        torch.cuda.synchronize()
        e.cache_append([a, b, c], 14, kv.data_ptr(), None)      # one page each
        e.cache_roll([a, b, c], 14)
        assert e.pool_info()[0] == 0
        with pytest.raises(ud.EngineError) as ei:
            e.cache_append([d], 14, kv.data_ptr(), None)
        assert ei.value.status == 5
        # a's next 14 frames need a second page: the batch fails as a whole and maps nothing
        with pytest.raises(ud.EngineError):
            e.cache_append([a, d], 14, kv.data_ptr(), None)
        assert e.pool_info()[0] == 0
        assert e.info(a)[:2] == (14, 14)
        e.close_stream(b)
        e.cache_append([d], 14, kv.data_ptr(), None)              # b's page is reusable
        e.synchronize()
    finally:
        e.close()
