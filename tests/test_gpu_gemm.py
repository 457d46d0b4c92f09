"""The MLA step's per-head contractions (k_b absorption, v_b) on the tcgen05
tensor cores with the 3xTF32 split, against a float64 reference and against
the CUDA-core f32 kernel.  The bound is f32-level: max |C - ref| / max |ref|
per head within 2e-5 (the 3xTF32 split drops A_lo*B_lo, ~2^-20 of a product,
and the lo parts keep 11 bits; the attention tolerance downstream is 1e-3)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    pool = kvcu.DevicePool(0, 1, 4, 16, 512, 64, True)
    yield kvcu, torch, pool
    pool.close()


def _run(kv, torch, pool, trans_b, heads, M, N, K, a_extra, impl):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + trans_b)
    # A rows as the step lays them out: [M][heads][K + a_extra]
    A = torch.randn((M, heads, K + a_extra), device="cuda", generator=g)
    if trans_b:
        B = torch.randn((heads, N, K), device="cuda", generator=g) / K ** 0.5
    else:
        B = torch.randn((heads, K, N), device="cuda", generator=g) / K ** 0.5
    C = torch.full((M, heads, N + 64), float("nan"), device="cuda")
    rc = kv.lib().kvcu_head_gemm(int(trans_b), heads, M, N, K, A.data_ptr(), heads * (K + a_extra), K + a_extra,
                                 B.data_ptr(), K if trans_b else N, N * K, C.data_ptr(), heads * (N + 64), N + 64,
                                 impl, pool.handle, None)
    assert rc == 0, kv.last_error()
    torch.cuda.synchronize()
    assert pool.status() == 0
    a64 = A[:, :, :K].double().permute(1, 0, 2)  # [heads][M][K]
    b64 = (B.double().transpose(1, 2) if trans_b else B.double())  # [heads][K][N]
    ref = torch.bmm(a64, b64).permute(1, 0, 2)  # [M][heads][N]
    got = C[:, :, :N].double()
    assert torch.isnan(C[:, :, N:]).all()  # nothing written past N
    err = ((got - ref).abs().amax(dim=(0, 2)) / ref.abs().amax(dim=(0, 2))).max().item()
    return C[:, :, :N].clone(), err


@pytest.mark.parametrize("trans_b,N,K,a_extra", [(False, 512, 128, 64), (True, 128, 512, 0)])
@pytest.mark.parametrize("M", [512, 200, 3])
def test_head_gemm_tensor_core_matches_f32(env, trans_b, N, K, a_extra, M):
    kv, torch, pool = env
    tc, e_tc = _run(kv, torch, pool, trans_b, 20, M, N, K, a_extra, 2)
    cc, e_cc = _run(kv, torch, pool, trans_b, 20, M, N, K, a_extra, 1)
    auto, _ = _run(kv, torch, pool, trans_b, 20, M, N, K, a_extra, 0)
    assert e_tc <= 2e-5, (e_tc, e_cc)
    assert e_cc <= 2e-5, (e_tc, e_cc)
    assert torch.equal(auto, tc)  # the default picks the tensor cores for these shapes


def test_head_gemm_tensor_core_refuses_other_shapes(env):
    kv, torch, pool = env
    A = torch.zeros((4, 2, 40), device="cuda")
    B = torch.zeros((2, 40, 96), device="cuda")
    C = torch.zeros((4, 2, 96), device="cuda")
    rc = kv.lib().kvcu_head_gemm(0, 2, 4, 96, 40, A.data_ptr(), 80, 40, B.data_ptr(), 96, 40 * 96, C.data_ptr(),
                                 192, 96, 2, pool.handle, None)
    assert rc == -16  # KVCU_ERR_UNSUPPORTED: N % 128 and K % 32
    rc = kv.lib().kvcu_head_gemm(0, 2, 4, 96, 40, A.data_ptr(), 80, 40, B.data_ptr(), 96, 40 * 96, C.data_ptr(),
                                 192, 96, 0, pool.handle, None)
    assert rc == 0  # the default falls back to the CUDA-core kernel
