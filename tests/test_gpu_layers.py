"""Several layers in one call (kvcu_mla_decode_layers, kvcu_append_layers and
the kvcache_* mirrors) against the same work done layer by layer.

With one one-layer plan repeated per layer, every work item of a multi-layer
launch computes exactly what the per-layer launch computes, so decode outputs
must be bit-identical; the appended Q8_0 bytes must be identical too (compared
in the checkpoint byte order).  A layered plan (kvcu_decode_plan_layers, which
the kvcache_* multi-layer calls use) cuts the sequences at other points, so a
split entry's partials are formed and merged differently: entries that no cut
splits stay bit-identical, split ones agree within the attention bound
(REL_TOL, max|diff| / max|row| per row)."""
import numpy as np
import pytest

from kvdata import REL_TOL, SCALE, W, rel_err_rows, seeded_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


def _pool(kv, torch, lens, bs, quant, nl, seed):
    nb = sum((int(L) + 1 + bs - 1) // bs for L in lens) + 4
    pool = kv.DevicePool(0, nl, nb, bs, 512, 64, quant)
    pool.zero()
    offs, tabs = seeded_tables([L + 1 for L in lens], bs, nb, seed)
    toff = torch.from_numpy(offs.astype(np.int32)).cuda()
    ttab = torch.from_numpy(tabs.astype(np.int32)).cuda()
    for layer in range(nl):
        kv.prefill_synthetic(pool, layer, lens, toff, ttab, seed, outlier_p=0.01)
    return pool, toff, ttab


@pytest.mark.parametrize("quant,bs,H", [(True, 64, 20), (True, 16, 8), (False, 16, 20)])
def test_decode_layers_matches_per_layer_calls(kv, quant, bs, H):
    import torch

    lens = [0, 1, 17, 130, 3000, 9000, 20000, 64, 700]
    nl, n = 3, len(lens)
    pool, toff, ttab = _pool(kv, torch, lens, bs, quant, nl, 71)
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn((nl, n, H, W), device="cuda", generator=torch.Generator(device="cuda").manual_seed(71))
    ws = kv.DecodeWorkspace(0, n, H, max_layers=nl)
    ws.plan(pool, lens_dev)
    want = torch.empty((nl, n, H, 512), device="cuda")
    for layer in range(nl):
        ws.decode(pool, layer, q[layer], toff, ttab, lens_dev, SCALE, want[layer])
    got = torch.full((nl, n, H, 512), float("nan"), device="cuda")
    ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, got)
    torch.cuda.synchronize()
    assert pool.status() == 0
    assert torch.equal(got, want)
    if quant:
        assert ws.last_launches == 2  # one decode launch + one combine for all layers
    # a sub-range of the pool's layers
    got2 = torch.full((2, n, H, 512), float("nan"), device="cuda")
    ws.decode_layers(pool, 1, q[1:].contiguous(), toff, ttab, lens_dev, SCALE, got2)
    torch.cuda.synchronize()
    assert torch.equal(got2, want[1:])
    ws.close()
    pool.close()


@pytest.mark.parametrize("lens,bs", [
    ([0, 1, 17, 130, 3000, 9000, 20000, 64, 700], 64),  # ragged, one empty entry
    ([3000] * 40 + [45000, 128, 129], 16),              # many cuts inside long entries
])
def test_decode_layers_with_a_layered_plan(kv, lens, bs):
    import torch

    nl, n, H = 4, len(lens), 20
    pool, toff, ttab = _pool(kv, torch, lens, bs, True, nl, 75)
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn((nl, n, H, W), device="cuda", generator=torch.Generator(device="cuda").manual_seed(75))
    ws = kv.DecodeWorkspace(0, n, H, max_layers=nl)
    ws.plan(pool, lens_dev)
    want = torch.empty((nl, n, H, 512), device="cuda")
    for layer in range(nl):
        ws.decode(pool, layer, q[layer], toff, ttab, lens_dev, SCALE, want[layer])
    ws.plan_layers(pool, lens_dev, nl)
    for rep in range(2):  # the plan serves repeated calls
        got = torch.full((nl, n, H, 512), float("nan"), device="cuda")
        ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, got)
        torch.cuda.synchronize()
        assert pool.status() == 0
        assert ws.last_launches == 2
        assert not torch.isnan(got).any(), rep
        err = rel_err_rows(got.cpu().numpy(), want.cpu().numpy())
        assert err <= REL_TOL, (rep, err)
        if 0 in lens:
            assert torch.all(got[:, lens.index(0)] == 0)
    # a layered plan serves only a decode of its own layer count
    with pytest.raises(kv.KVCudaError):
        ws.decode(pool, 0, q[0], toff, ttab, lens_dev, SCALE, got[0])
    with pytest.raises(kv.KVCudaError):
        ws.decode_layers(pool, 0, q[:2].contiguous(), toff, ttab, lens_dev, SCALE, got[:2].contiguous())
    with pytest.raises(kv.KVCudaError):
        ws.plan_layers(pool, lens_dev, nl + 1)  # more layers than the workspace holds
    # a one-layer plan again: per-layer decodes, bit-identical to before
    ws.plan(pool, lens_dev)
    again = torch.empty((n, H, 512), device="cuda")
    ws.decode(pool, 2, q[2], toff, ttab, lens_dev, SCALE, again)
    torch.cuda.synchronize()
    assert torch.equal(again, want[2])
    ws.close()
    pool.close()


def test_layered_plan_is_refused_on_the_cuda_core_path(kv):
    import torch

    lens = [100, 2000]
    pool, toff, ttab = _pool(kv, torch, lens, 16, False, 2, 76)  # f32 pool: CUDA-core decode
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = kv.DecodeWorkspace(0, 2, 8, max_layers=2)
    ws.plan_layers(pool, lens_dev, 2)
    q = torch.zeros((2, 2, 8, W), device="cuda")
    out = torch.zeros((2, 2, 8, 512), device="cuda")
    with pytest.raises(kv.KVCudaError):
        ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, out)
    ws.plan(pool, lens_dev)
    ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, out)  # a one-layer plan works
    torch.cuda.synchronize()
    assert pool.status() == 0
    ws.close()
    pool.close()


def test_decode_refuses_a_batch_other_than_the_planned_one(kv):
    import torch

    lens = [100, 200, 300]
    pool, toff, ttab = _pool(kv, torch, lens, 16, True, 2, 77)
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = kv.DecodeWorkspace(0, 3, 8, max_layers=2)
    q = torch.zeros((2, 3, 8, W), device="cuda")
    out = torch.zeros((2, 3, 8, 512), device="cuda")
    with pytest.raises(kv.KVCudaError):  # no plan yet
        ws.decode(pool, 0, q[0], toff, ttab, lens_dev, SCALE, out[0])
    ws.plan(pool, lens_dev)
    with pytest.raises(kv.KVCudaError):  # two entries against a plan of three
        ws.decode(pool, 0, q[0, :2].contiguous(), toff, ttab, lens_dev, SCALE, out[0, :2].contiguous())
    with pytest.raises(kv.KVCudaError):
        ws.decode_layers(pool, 0, q[:, :2].contiguous(), toff, ttab, lens_dev, SCALE, out[:, :2].contiguous())
    ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, out)  # the planned batch
    torch.cuda.synchronize()
    assert pool.status() == 0
    ws.close()
    pool.close()


def test_decode_layers_needs_a_workspace_with_room_for_the_layers(kv):
    import torch

    lens = [100, 200]
    pool, toff, ttab = _pool(kv, torch, lens, 16, True, 2, 72)
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = kv.DecodeWorkspace(0, 2, 8)  # one layer of partials
    ws.plan(pool, lens_dev)
    q = torch.zeros((2, 2, 8, W), device="cuda")
    out = torch.zeros((2, 2, 8, 512), device="cuda")
    with pytest.raises(kv.KVCudaError):
        ws.decode_layers(pool, 0, q, toff, ttab, lens_dev, SCALE, out)
    with pytest.raises(kv.KVCudaError) as e:
        ws.decode_layers(pool, 1, q, toff, ttab, lens_dev, SCALE, out)  # layers 1..2 of a 2-layer pool
    assert e.value.name == "LayerOutOfBounds"
    ws.close()
    pool.close()


@pytest.mark.parametrize("quant", [True, False])
def test_append_layers_matches_per_layer_appends(kv, quant):
    import torch

    lens = [5, 64, 129, 1000]
    nl, n = 4, len(lens)
    pools = [_pool(kv, torch, lens, 16, quant, nl, 73) for _ in range(2)]
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    seq = torch.arange(n, dtype=torch.int32, device="cuda")
    rows = torch.randn((nl, n, W), device="cuda", generator=torch.Generator(device="cuda").manual_seed(73)) * 3
    lens_a = torch.tensor(lens, dtype=torch.int32, device="cuda")
    lens_b = lens_a.clone()
    (pa, toff, ttab), (pb, toff_b, ttab_b) = pools
    for layer in range(nl):
        pa.append(layer, rows[layer], seq, pos, toff, ttab, lens=lens_a)
    pb.append_layers(0, rows, seq, pos, toff_b, ttab_b, lens=lens_b)
    torch.cuda.synchronize()
    assert pa.status() == 0 and pb.status() == 0
    assert pa.read_checkpoint() == pb.read_checkpoint()
    assert torch.equal(lens_a, lens_b) and torch.equal(lens_b.cpu(), torch.tensor(lens) + 1)
    pa.close()
    pb.close()


@pytest.mark.parametrize("host_io", [0, 1, 2])  # q / out in place over PCIe, DMA copies, q by DMA
def test_append_decode_layers_host_buffers_match_per_layer_calls(kv, host_io):
    import torch

    lens = [40, 300, 5000, 12000, 3]
    nl, n, H = 3, len(lens), 20
    caches = []
    for _ in range(2):
        nb = sum((L + 8 + 63) // 64 for L in lens) + 8
        c = kv.KVCache.with_blocks(nl, 512, 64, nb, block_size=64, quantized=True)
        for _ in range(n - 1):
            c.seq_create()
        ids = np.arange(n, dtype=np.uint32)
        for i in range(n):
            c.seq_ensure_capacity(i, lens[i] + 4)
        for layer in range(nl):
            c.prefill_synthetic(layer, ids, lens, 74, 0.01)
        caches.append(c)
    torch.cuda.synchronize()
    g = torch.Generator().manual_seed(74)
    for step in range(2):
        pos = (np.array(lens) + step).astype(np.uint32)
        rows = torch.randn((nl, n, W), generator=g).pin_memory()
        q = torch.randn((nl, n, H, W), generator=g).pin_memory()
        want = torch.empty((nl, n, H, 512)).pin_memory()
        got = torch.full((nl, n, H, 512), float("nan")).pin_memory()
        a, b = caches
        for layer in range(nl):
            a.appendBatch(layer, ids, pos, rows[layer].numpy())
            a.mlaDecode_ptr(layer, n, ids, q[layer].data_ptr(), H, SCALE, want[layer].data_ptr())
        b.set_host_io(host_io)
        b.appendDecodeLayers_ptr(0, nl, n, ids, pos, rows.data_ptr(), q.data_ptr(), H, SCALE, got.data_ptr())
        assert b.last_decode_mapped == (host_io != kv.KVCache.HOST_IO_COPY)
        assert not torch.isnan(got).any(), step
        err = rel_err_rows(got.numpy(), want.numpy())  # layered plan against per-layer plans
        assert err <= REL_TOL, (step, err)
        assert all(b.seq_len(i) == a.seq_len(i) == lens[i] + step + 1 for i in range(n))
    for c in caches:
        c.close()
