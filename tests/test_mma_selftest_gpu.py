"""The tcgen05 layer (SW128 operand images, smem/instruction descriptors,
M=64 / M=128 TMEM layouts, A read from TMEM, bf16 / fp16 / tf32 kinds)
against torch matmul, for every shape the prefill kernels issue."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [  # (kind, M, N, K[, flags]): shapes the prefill kernels issued in this and earlier designs
    ("bf16", 128, 64, 128),   # [K;Q] K^T
    ("tf32", 64, 64, 64),     # Neumann products
    ("tf32", 64, 256, 64),    # [W | U]
    ("tf32", 64, 16, 128),    # W S^T, BV=16
    ("tf32", 64, 32, 128),    # W S^T, BV=32
    ("bf16", 64, 16, 128),    # Q S^T
    ("bf16", 64, 32, 128),
    ("tf32", 128, 16, 64),    # (tail K)^T Delta
    ("tf32", 128, 32, 64),
    ("bf16", 64, 16, 64),     # P Delta
    ("bf16", 64, 32, 64),
    ("tf32", 128, 128, 128),
    ("bf16", 128, 256, 128),
    # MN-major operands and the lane-16 accumulator of a packed M=64 pair
    ("tf32", 64, 64, 64, 2),
    ("tf32", 64, 64, 64, 1),
    ("tf32", 64, 64, 64, 3),
    ("tf32", 128, 32, 64, 2),
    ("tf32", 128, 16, 64, 1),
    ("tf32", 128, 128, 64, 3),
    ("bf16", 64, 128, 64, 2),
    ("bf16", 128, 64, 64, 1),
    ("bf16", 128, 256, 64, 3),
    ("tf32", 64, 64, 64, 4),
    ("tf32", 64, 256, 64, 6),
    ("bf16", 64, 128, 64, 7),
    ("tf32", 128, 32, 128, 2),
    ("bf16", 64, 64, 128, 2),
    # fp16 operands (kind::f16 with format F16)
    ("f16", 128, 64, 128),
    ("f16", 64, 64, 64, 2),
    ("f16", 128, 128, 64, 3),
    ("f16", 64, 256, 64, 6),
    ("f16", 128, 64, 128, 2),
    # A operand in TMEM (the carry's state and output MMAs)
    ("f16", 128, 128, 128, 8),
    ("f16", 128, 64, 128, 8),
    ("f16", 128, 128, 64, 10),
    ("bf16", 128, 64, 64, 8),
]


def _tf32(x):
    """Round-to-nearest (ties away) to tf32, as cvt.rna.tf32.f32."""
    xi = x.contiguous().view(torch.int32)
    return ((xi + 0x1000) & ~0x1FFF).view(torch.float32)


@pytest.mark.parametrize("case", SHAPES, ids=lambda c: "-".join(map(str, c)))
def test_mma_selftest(pkg, cuda_dev, case):
    kind, M, N, K = case[:4]
    flags = case[4] if len(case) > 4 else 0
    C = pkg._capi
    lib = C.load()
    g = torch.Generator().manual_seed(M * 1000 + N + K)
    A = torch.randn(M, K, generator=g)
    B = torch.randn(N, K, generator=g)
    if kind in ("bf16", "f16"):
        dt = torch.bfloat16 if kind == "bf16" else torch.float16
        A, B = A.to(dt), B.to(dt)
        ref = A.double() @ B.double().T
        code = C.MMA_KIND_BF16 if kind == "bf16" else C.MMA_KIND_F16
    else:
        ref = _tf32(A).double() @ _tf32(B).double().T
        code = C.MMA_KIND_TF32
    dA, dB = A.to(cuda_dev), B.to(cuda_dev)
    D = torch.full((M, N), float("nan"), device=cuda_dev)
    rc = lib.gdn_mma_selftest(code, flags, M, N, K, ctypes.c_void_p(dA.data_ptr()), ctypes.c_void_p(dB.data_ptr()),
                              ctypes.c_void_p(D.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, C.status_string(rc)
    torch.cuda.synchronize()
    assert pkg.prefill.device_status(cuda_dev) == 0
    err = (D.double().cpu() - ref).abs().max().item()
    assert err < 1e-3 * max(1.0, ref.abs().max().item()), f"max err {err}"


def test_mma_selftest_rejects_partial_mn_rows(pkg, cuda_dev):
    """MN-major images must fill whole 128-byte rows (bf16 N=32 would not)."""
    lib = pkg._capi.load()
    buf = torch.zeros(64 * 128, device=cuda_dev)
    p = ctypes.c_void_p(buf.data_ptr())
    assert lib.gdn_mma_selftest(pkg._capi.MMA_KIND_BF16, 2, 64, 32, 128, p, p, p, None) == 2


def test_bounded_wait_expires_and_unwinds(pkg, cuda_dev):
    """A wait that nothing completes: the self-test kernel issues no MMA and
    never signals its barrier (GDN_MMA_NO_COMPLETION).  The kernel's bounded
    wait gives up after its time limit (10 ms), the device status word reports
    GDN_ERR_DEVICE_TIMEOUT, D stays unwritten, and the kernel releases its TMEM:
    the context stays usable and the next tensor-core kernel runs normally."""
    import time

    C = pkg._capi
    lib = C.load()
    pkg.prefill.device_status(cuda_dev)  # clear
    A = torch.randn(128, 64).to(torch.bfloat16).to(cuda_dev)
    B = torch.randn(64, 64).to(torch.bfloat16).to(cuda_dev)
    D = torch.full((128, 64), float("nan"), device=cuda_dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    assert lib.gdn_mma_selftest(C.MMA_KIND_BF16, C.MMA_NO_COMPLETION, 128, 64, 64, P(A), P(B), P(D), stream) == 0
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert pkg.prefill.device_status(cuda_dev) == C.GDN_ERR_DEVICE_TIMEOUT
    assert torch.isnan(D).all()
    assert took < 2.0, f"the expired wait took {took:.3f} s"
    # TMEM was released: the same kernel allocates it again and completes normally
    assert lib.gdn_mma_selftest(C.MMA_KIND_BF16, 0, 128, 64, 64, P(A), P(B), P(D), stream) == 0
    torch.cuda.synchronize()
    assert pkg.prefill.device_status(cuda_dev) == 0
    ref = A.double().cpu() @ B.double().cpu().T
    assert (D.double().cpu() - ref).abs().max().item() < 1e-3 * ref.abs().max().item()
