"""The tcgen05 NVFP4 GEMM against fp64 dequantise-then-matmul of the same NVFP4 operands.

Operands are quantised on the device (bit-exact with the oracle, tests/test_quant_gpu.py) and dequantised on the
CPU by the oracle.  GEMM outputs are bf16 (as TensorFold's prompt GEMM returns, tfvideo/linear.py:151), so the
reference is bf16(fp64 result) and the bar is rel-L2 <= 1e-3.  Fused epilogues are checked against the oracle's
gate_add / gelu / swiglu / quantiser applied to that reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ON
from oracle import ops as OO

from helpers import bf16_array, device_ok, need_gpu, to_dev, to_np, u8

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(autouse=True)
def _gpu():
    need_gpu()


def _linear(N_, K_, seed, interleave=False, bias=None):
    from tfvideo import linear as L

    w = bf16_array((N_, K_), seed, scale=0.02, outliers=False)
    lin = L.Nvfp4Linear(to_dev(w), interleave16=interleave, bias=bias)
    B = ON.dequantize(u8(lin.codes), ON.sf_from_tiled(u8(lin.sf), N_, K_ // 16), lin.g).astype(np.float64)
    return lin, B


def _input(M, K_, seed, lin):
    from tfvideo import linear as L

    x = bf16_array((M, K_), seed)
    g = ON.global_scale(float(np.abs(x).max()))
    lin.set_act(float(g))
    codes, sf = L.quantize(to_dev(x), g=float(g), tiled=True)
    A = ON.dequantize(u8(codes), ON.sf_from_tiled(u8(sf), M, K_ // 16), g).astype(np.float64)
    return codes, sf, A


def _epi(**kw):
    from tfvideo import native as N
    return N.H3Epilogue(**kw)


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 384, 768), (1000, 512, 2048), (37, 1536, 5120),
                                   (4096, 256, 5120)])
def test_gemm_store(M, N, K):
    from tfvideo import native as Nat

    lin, B = _linear(N, K, seed=N + K)
    codes, sf, A = _input(M, K, seed=M, lin=lin)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    lin.gemm(codes, sf, M, _epi(kind=Nat.H3_EPI_STORE, out=out.data_ptr(), ldo=N))
    ref = ON.bf16_round((A @ B.T).astype(np.float32))
    assert OO.rel_l2(to_np(out), ref) <= TOL
    device_ok()


def test_gemm_bias_and_reference_call():
    """Nvfp4Linear.__call__ (dynamic per-call scale, as the reference's first forward) with a fused fp32 bias."""

    from tfvideo import linear as L

    M, N, K = 200, 512, 1024
    bias = np.random.RandomState(2).randn(N).astype(np.float32)
    w = bf16_array((N, K), 21, scale=0.02, outliers=False)
    lin = L.Nvfp4Linear(to_dev(w), bias=torch.from_numpy(bias))
    x = bf16_array((M, K), 22)
    y = to_np(lin(to_dev(x)))
    ref = OO.linear_nvfp4(x, (u8(lin.codes), ON.sf_from_tiled(u8(lin.sf), N, K // 16), np.float32(lin.g)),
                          bias=bias)
    assert OO.rel_l2(y, ref) <= TOL
    device_ok()


@pytest.mark.parametrize("part", [0, 1])
def test_gemm_gate_residual(part):
    from tfvideo import native as Nat

    M, N, K = 300, 512, 1024
    lin, B = _linear(N, K, seed=5)
    codes, sf, A = _input(M, K, seed=6, lin=lin)
    rs = np.random.RandomState(7)
    mod = (0.1 * rs.randn(4, 6, N)).astype(np.float32)
    idx = rs.randint(0, 4, size=M).astype(np.int32)
    x = bf16_array((M, N), 8)
    xt, modt, idxt = to_dev(x), to_dev(mod, torch.float32), to_dev(idx, torch.int32)
    lin.gemm(codes, sf, M, _epi(kind=Nat.H3_EPI_GATE_RESID, x=xt.data_ptr(), ldx=N, mod=modt.data_ptr(),
                                idx=idxt.data_ptr(), gate_part=part))
    y = ON.bf16_round((A @ B.T).astype(np.float32))
    ref = OO.gate_add(x, y, mod, part, idx)
    got = to_np(xt)
    # y may differ from the reference by one bf16 ulp where the fp64 result sits near a rounding boundary; that
    # moves x + y * gate by at most |gate| * ulp(y) before x's own rounding
    g = mod[idx, 3 * part + 2]
    bound = 2.0 ** -7 * (np.abs(ref) + np.abs(y * g)) + 1e-30
    assert (np.abs(got - ref) <= bound).all()
    assert (got == ref).mean() > 0.98
    assert OO.rel_l2(got - x, ref - x) <= 2e-2
    device_ok()


@pytest.mark.parametrize("act", ["gelu", "swiglu"])
@pytest.mark.parametrize("quant", [False, True])
def test_gemm_activation_epilogues(act, quant):
    """fc1's epilogue: activation in bf16 (+ NVFP4 for fc2).  The quantised form must equal the oracle quantiser on
    the epilogue's own bf16 activation, bit for bit, and the amax slot must hold its max |a|."""

    from tfvideo import linear as L
    from tfvideo import native as Nat

    M, N, K = 260, 1024, 512
    lin, B = _linear(N, K, seed=31, interleave=(act == "swiglu"))
    codes, sf, A = _input(M, K, seed=32, lin=lin)
    y = ON.bf16_round((A @ B.T).astype(np.float32))
    if act == "swiglu":     # undo the 16-row interleave of the weight: [g0..g15, u0..u15, g16..]
        yi = y.reshape(M, N // 32, 2, 16)
        ref = OO.swiglu(np.concatenate([yi[:, :, 0].reshape(M, -1), yi[:, :, 1].reshape(M, -1)], 1))
    else:
        ref = OO.gelu_tanh(y)
    F = ref.shape[1]
    kind = Nat.ACT_SWIGLU if act == "swiglu" else Nat.ACT_GELU
    out = torch.empty((M, F), dtype=torch.bfloat16, device="cuda")
    qs = L.new_slots(1, "cuda")
    if quant:
        g = ON.global_scale(float(np.abs(ref).max()))
        qs[0, 1] = float(g)
        qc = torch.empty((M, F // 2), dtype=torch.uint8, device="cuda")
        qsf = torch.zeros(Nat.sf_tiled_bytes(M, F), dtype=torch.uint8, device="cuda")
        lin.gemm(codes, sf, M, _epi(kind=Nat.H3_EPI_ACT_Q, act_kind=kind, out=out.data_ptr(), ldo=F,
                                    qcodes=qc.data_ptr(), qsf=qsf.data_ptr(), q_slot=Nat.slot_ptr(qs, 0)))
    else:
        lin.gemm(codes, sf, M, _epi(kind=Nat.H3_EPI_ACT_BF16, act_kind=kind, out=out.data_ptr(), ldo=F,
                                    q_slot=Nat.slot_ptr(qs, 0)))
    a = to_np(out)
    assert OO.rel_l2(a, ref) <= 5e-3
    assert to_np(qs)[0, 0] == np.abs(a).max()
    if quant:
        rc, rsf = ON.quantize(a, g)
        assert np.array_equal(u8(qc), rc)
        assert np.array_equal(ON.sf_from_tiled(u8(qsf), M, F // 16), rsf)
    device_ok()


def test_gemm_rejects_bad_shapes():
    from tfvideo import native as Nat

    lin, _ = _linear(256, 256, seed=1)
    codes = torch.zeros((64, 64), dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="K % 256"):
        Nat.gemm_nvfp4(codes, codes, lin.slot_ptr(), lin.codes, lin.sf, lin.g, 64, 256, 128,
                       _epi(kind=Nat.H3_EPI_STORE, out=codes.data_ptr(), ldo=256))
