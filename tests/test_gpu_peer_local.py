"""The head-sharded gather protocol and its bounded peer wait, on one GPU.

tl_debug_peer_attach lets a device region of this process stand in for the
other rank's CUDA-IPC region ([flags 256 B][gathered outputs]), so one GPU
can play rank 0 of a world of 2:
  * a "peer" that has published (its flag holds the epoch) has its slice
    pulled into this rank's gather area next to this rank's own decode
    output, which matches the fp64 oracle;
  * a "peer" that never publishes makes the kernel's flag wait run out
    after the short limit set with tl_set_peer_wait_limit: the call returns,
    tl_sync_check reports TL_ERR_DEVICE_FAULT ("bounded wait timed out"),
    and the handle keeps decoding correctly afterwards.
Failure is made on the host side (a flag that nothing sets); no fault, trap
or endless wait is involved.
"""
import math
import time

import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import Run, check_close, d2h, to_dev

pytestmark = pytest.mark.gpu

L, Hq, Hkv, D, bs = 2, 8, 2, 128, 16  # rank 0's slice of a 2-way head shard
LENS = [37, 300, 129]


@pytest.fixture
def setup():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    import torch

    r = Run.create(L=L, Hq=Hq, Hkv=Hkv, D=D, bs=bs, max_seq_len=512, max_batch=len(LENS))
    sids = [r.allocate(512) for _ in LENS]
    for i, (sid, P) in enumerate(zip(sids, LENS)):
        r.prefill(sid, P, seed=70 + i)
    slice_bytes = len(sids) * Hq * D * 2
    gather_bytes = L * 2 * slice_bytes
    r.cache.peer_init(0, 2, gather_bytes)
    fake = torch.zeros(256 + gather_bytes, dtype=torch.uint8, device="cuda")
    assert fake.data_ptr() % 256 == 0
    r.cache.debug_peer_attach(1, fake.data_ptr())
    yield r, sids, fake, slice_bytes
    r.cache.close()


def _expected(r, sids, q, layer):
    return np.stack([O.decode_one(q[i], np.stack(r.logical_k[(s, layer)]), np.stack(r.logical_v[(s, layer)]),
                                  1.0 / math.sqrt(D)) for i, s in enumerate(sids)])


def test_published_peer_slice_is_pulled(setup):
    import torch

    r, sids, fake, slice_bytes = setup
    layer, epoch = 1, 5
    off = layer * 2 * slice_bytes
    peer_slice = O.normal_f16((len(sids), Hq, D), 4242)
    fake[256 + off + slice_bytes: 256 + off + 2 * slice_bytes] = \
        torch.from_numpy(peer_slice.view(np.uint8).reshape(-1)).cuda()
    fake[4:8] = torch.tensor([epoch], dtype=torch.int32).view(torch.uint8).cuda()  # rank 1's flag
    q = O.normal_f16((len(sids), Hq, D), 31)
    qd = to_dev(q)
    r.cache.decode_attention_peer(layer, qd.data_ptr(), sids, off, epoch)
    r.cache.sync_check()
    g, _ = r.cache.peer_buffer()
    n = slice_bytes // 2
    own = O.f16_to_f32(d2h(g + off, n).reshape(len(sids), Hq, D))
    pulled = d2h(g + off + slice_bytes, n).reshape(len(sids), Hq, D)
    check_close(own, _expected(r, sids, q, layer), "rank 0's own slice")
    assert np.array_equal(pulled, peer_slice), "rank 1's slice was not pulled intact"
    assert int(d2h(g - 256, 2, np.uint32)[0]) == epoch, "rank 0 did not publish its epoch"


def test_unpublished_peer_wait_runs_out_and_handle_stays_usable(setup):
    import torch

    r, sids, fake, slice_bytes = setup
    r.cache.set_peer_wait_limit(0.05)
    q = O.normal_f16((len(sids), Hq, D), 32)
    qd = to_dev(q)
    t0 = time.time()
    r.cache.decode_attention_peer(0, qd.data_ptr(), sids, 0, 1)  # flag of rank 1 stays 0
    with pytest.raises(T.DeviceFault) as e:
        r.cache.sync_check()
    elapsed = time.time() - t0
    assert "bounded wait timed out" in str(e.value)
    assert elapsed < 5.0, f"the 50 ms wait took {elapsed:.1f} s to give up"
    # the handle still decodes, plainly and in peer mode once the peer publishes
    r.decode_and_check(0, sids, seed=33)
    r.decode_and_check(1, sids, seed=34)
    fake[4:8] = torch.tensor([2], dtype=torch.int32).view(torch.uint8).cuda()
    r.cache.decode_attention_peer(0, qd.data_ptr(), sids, 0, 2)
    r.cache.sync_check()
    g, _ = r.cache.peer_buffer()
    own = O.f16_to_f32(d2h(g, slice_bytes // 2).reshape(len(sids), Hq, D))
    check_close(own, _expected(r, sids, q, 0), "peer-mode decode after the timeout")
