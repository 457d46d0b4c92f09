"""kvcu_mla_decode_noalloc -- the decode entry point that allocates nothing --
against kvcu_decode_plan + kvcu_mla_decode on the same pool and queries.

Called through the C-ABI (ctypes on libkvcuda.so).  Each case runs the
no-allocation entry point twice in a row (the fixed scratch is reused by the
second call) and compares both outputs with the workspace path.  The file is
named to be collected last, so in a full run it also exercises the scratch
after every other GPU test has used the library in the same process."""
import numpy as np
import pytest

from kvdata import REL_TOL, SCALE, W, rel_err_rows, seeded_tables

pytestmark = pytest.mark.gpu

ERR_INVALID_ARG = -11


@pytest.fixture(scope="module")
def torch():
    import torch as t

    if not t.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    return t


@pytest.fixture(scope="module")
def kv(torch):
    import kvcu

    kvcu.init(0)
    return kvcu


def _noalloc(kv, pool, layer, n, n_seqs, toff, tabs, lens, q, n_heads, out, seq_ids=None):
    ptr = lambda t: None if t is None else t.data_ptr()
    return kv.lib().kvcu_mla_decode_noalloc(pool.handle, layer, n, ptr(seq_ids), n_seqs, ptr(toff),
                                            ptr(tabs), ptr(lens), ptr(q), n_heads, SCALE, ptr(out),
                                            None)


def _build(kv, torch, lens, bs, quant, n_layers, seed):
    dev = torch.device("cuda", 0)
    nb = sum((int(L) + bs - 1) // bs for L in lens) + 4
    pool = kv.DevicePool(0, n_layers, nb, bs, 512, 64, quant)
    pool.zero()
    offs, tabs = seeded_tables(lens, bs, nb, seed)
    toff = torch.from_numpy(offs.astype(np.int32)).to(dev)
    ttab = torch.from_numpy(tabs.astype(np.int32)).to(dev)
    lens_dev = torch.from_numpy(np.asarray(lens, np.int32)).to(dev)
    for layer in range(n_layers):
        kv.prefill_synthetic(pool, layer, lens, toff, ttab, seed, outlier_p=0.01)
    torch.cuda.synchronize()
    return pool, toff, ttab, lens_dev


def _compare(kv, torch, lens, bs, quant, n_heads, seed, n_layers=2, seq_ids=None):
    dev = torch.device("cuda", 0)
    pool, toff, ttab, lens_dev = _build(kv, torch, lens, bs, quant, n_layers, seed)
    ids = None if seq_ids is None else torch.from_numpy(np.asarray(seq_ids, np.int32)).to(dev)
    n = len(lens) if seq_ids is None else len(seq_ids)
    ws = kv.DecodeWorkspace(0, n, n_heads)
    gen = torch.Generator(device=dev).manual_seed(seed)
    for layer in range(n_layers):
        q = torch.randn((n, n_heads, W), device=dev, generator=gen)
        want = torch.empty((n, n_heads, 512), device=dev)
        ws.plan(pool, lens_dev, seq_ids=ids, n=n)
        ws.decode(pool, layer, q, toff, ttab, lens_dev, SCALE, want, seq_ids=ids)
        outs = []
        for _ in range(2):
            got = torch.full((n, n_heads, 512), float("nan"), device=dev)
            rc = _noalloc(kv, pool, layer, n, len(lens), toff, ttab, lens_dev, q, n_heads, got, ids)
            assert rc == 0, kv.last_error()
            outs.append(got)
        torch.cuda.synchronize()
        assert pool.status() == 0
        w = want.cpu().numpy()
        for got in outs:
            g = got.cpu().numpy()
            assert np.isfinite(g).all()
            assert rel_err_rows(g, w) <= REL_TOL, (layer, rel_err_rows(g, w))
        # the same inputs give the same bits on the second call
        assert torch.equal(outs[0], outs[1])
    ws.close()
    pool.close()


def test_noalloc_q8_tensor_core_split_sequences(kv, torch):
    # long sequences are split into several work items (partials + combine)
    _compare(kv, torch, [1, 130, 4000, 9000, 20000, 0, 77], 64, True, 20, 901)


def test_noalloc_f32_cuda_core(kv, torch):
    _compare(kv, torch, [3, 500, 2500, 0, 1200], 16, False, 8, 902)


def test_noalloc_max_batch_with_seq_ids(kv, torch):
    rng = np.random.default_rng(903)
    lens = rng.integers(0, 3000, 70).tolist()
    ids = rng.permutation(70)[:64].tolist()  # KVCU_NOALLOC_MAX_BATCH entries
    _compare(kv, torch, lens, 32, True, 16, 903, n_layers=1, seq_ids=ids)


def test_noalloc_leaves_free_device_memory_unchanged(kv, torch):
    # The point of the entry point: after kvcu_init (which reserves the fixed
    # scratch) and one warm-up call (which lets CUDA load the kernels it
    # launches), repeated calls take no device memory at all.
    dev = torch.device("cuda", 0)
    lens = [5, 300, 7000, 16000, 0, 900]
    pool, toff, ttab, lens_dev = _build(kv, torch, lens, 64, True, 1, 905)
    n, H = len(lens), 20
    q = torch.randn((n, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(905))
    out = torch.empty((n, H, 512), device=dev)
    assert _noalloc(kv, pool, 0, n, n, toff, ttab, lens_dev, q, H, out) == 0, kv.last_error()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    for _ in range(5):
        assert _noalloc(kv, pool, 0, n, n, toff, ttab, lens_dev, q, H, out) == 0, kv.last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert pool.status() == 0
    pool.close()


def test_noalloc_on_two_devices_from_one_process(kv, torch):
    # Kernel set-up (dynamic shared memory limits) and the scratch address are
    # per device; one process drives both GPUs in turn.
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lens = [40, 2500, 9000, 130]
    n, H = len(lens), 20
    for d in (1, 0, 1):
        dev = torch.device("cuda", d)
        kv.init(d)
        nb = sum((L + 63) // 64 for L in lens) + 4
        pool = kv.DevicePool(d, 1, nb, 64, 512, 64, True)
        pool.zero()
        offs, tabs = seeded_tables(lens, 64, nb, 906 + d)
        toff = torch.from_numpy(offs.astype(np.int32)).to(dev)
        ttab = torch.from_numpy(tabs.astype(np.int32)).to(dev)
        lens_dev = torch.from_numpy(np.asarray(lens, np.int32)).to(dev)
        with torch.cuda.device(d):
            kv.prefill_synthetic(pool, 0, lens, toff, ttab, 906, outlier_p=0.01)
            q = torch.randn((n, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(d))
            want = torch.empty((n, H, 512), device=dev)
            got = torch.full((n, H, 512), float("nan"), device=dev)
            ws = kv.DecodeWorkspace(d, n, H)
            ws.plan(pool, lens_dev)
            ws.decode(pool, 0, q, toff, ttab, lens_dev, SCALE, want)
            assert _noalloc(kv, pool, 0, n, n, toff, ttab, lens_dev, q, H, got) == 0, kv.last_error()
            torch.cuda.synchronize(dev)
        assert pool.status() == 0
        assert rel_err_rows(got.cpu().numpy(), want.cpu().numpy()) <= REL_TOL
        ws.close()
        pool.close()


def test_noalloc_rejects_sizes_beyond_the_scratch(kv, torch):
    dev = torch.device("cuda", 0)
    pool, toff, ttab, lens_dev = _build(kv, torch, [10] * 66, 16, True, 1, 904)
    q = torch.zeros((66, 33, W), device=dev)
    out = torch.full((66, 33, 512), 7.0, device=dev)
    assert _noalloc(kv, pool, 0, 65, 66, toff, ttab, lens_dev, q, 20, out) == ERR_INVALID_ARG
    assert "65" in kv.last_error()
    assert _noalloc(kv, pool, 0, 8, 66, toff, ttab, lens_dev, q, 33, out) == ERR_INVALID_ARG
    assert _noalloc(kv, pool, 0, 8, 66, toff, ttab, lens_dev, q, 0, out) == ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
    pool.close()
