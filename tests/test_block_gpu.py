"""End-to-end transformer block through the library (grxDNN + grxBLAS), the
gate the reference's roadmap sets for grxDNN ("attention + GEMM + layernorm +
softmax end-to-end vs a PyTorch CPU reference", docs/designs/grxcp_roadmap.md:
874-876), checked against an fp64 CPU chain built from the oracle.

Row-major activations [T, H]; a linear layer y = x W^T + b is one GemmEx with
C = W^T-as-stored times x: transa = T on W [out, in], transb = N on x, bias over
the rows of C (the output features), residuals as beta = 1 with C preloaded.
The attention reads Q, K, V straight out of the fused QKV buffer by stride.
The CPU chain rounds to bf16 where the GPU stores bf16, so the comparison
measures the kernels, not the storage format."""
import math

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N
from grxcp_b200 import blas as Bl
from grxcp_b200 import dnn as D
from grxcp_b200.dnn import attn_desc

pytestmark = pytest.mark.gpu


def bf(x):
    return oracle.round_to("bf16", np.asarray(x, np.float32))


def test_transformer_block_end_to_end():
    torch.cuda.set_device(0)
    rng = np.random.default_rng(0)
    Bt, S, H, heads, F = 2, 256, 1024, 8, 4096
    Dh = H // heads
    T = Bt * S
    x = bf(rng.standard_normal((T, H)))
    w = {n: bf(rng.standard_normal(shape) / math.sqrt(shape[1])) for n, shape in
         [("qkv", (3 * H, H)), ("o", (H, H)), ("up", (F, H)), ("down", (H, F))]}
    b = {n: (rng.standard_normal(k) * 0.02).astype(np.float32) for n, k in
         [("qkv", 3 * H), ("o", H), ("up", F), ("down", H)]}
    g1, be1 = (1 + 0.02 * rng.standard_normal(H)).astype(np.float32), (0.02 * rng.standard_normal(H)).astype(np.float32)
    g2, be2 = (1 + 0.02 * rng.standard_normal(H)).astype(np.float32), (0.02 * rng.standard_normal(H)).astype(np.float32)

    dev = lambda a, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(dt)  # noqa
    dx = dev(x)
    dw = {n: dev(v) for n, v in w.items()}
    db = {n: dev(v, torch.float32) for n, v in b.items()}
    dg1, dbe1, dg2, dbe2 = (dev(v, torch.float32) for v in (g1, be1, g2, be2))
    bh, dh = Bl.Handle(), D.Handle()

    def linear(inp, name, out, beta=0.0, act=N.ACT_NONE):
        o_feat, i_feat = w[name].shape
        assert bh.set_epilogue(bias=db[name], bias_type=N.GRX_R_32F, bias_over_rows=True, activation=act) == 0
        assert bh.gemm_ex(N.OP_T, N.OP_N, o_feat, T, i_feat, 1.0, dw[name], N.GRX_R_16BF, i_feat, inp, N.GRX_R_16BF,
                          i_feat, beta, out, N.GRX_R_16BF, o_feat) == N.SUCCESS

    h1 = torch.empty_like(dx)
    assert dh.layernorm(dx, dg1, dbe1, 1e-5, h1) == N.SUCCESS
    qkv = torch.empty(T, 3 * H, device="cuda", dtype=torch.bfloat16)
    linear(h1, "qkv", qkv)
    attn = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    q_desc = attn_desc(None, Bt, heads, S, Dh)
    q_desc.strideBatch, q_desc.strideHead, q_desc.strideSeq = S * 3 * H, Dh, 3 * H
    k_desc = attn_desc(None, Bt, heads, S, Dh)
    k_desc.strideBatch, k_desc.strideHead, k_desc.strideSeq = S * 3 * H, Dh, 3 * H
    o_desc = attn_desc(None, Bt, heads, S, Dh)
    o_desc.strideBatch, o_desc.strideHead, o_desc.strideSeq = S * H, Dh, H
    base = qkv.data_ptr()
    assert dh.attention(base, base + 2 * H, base + 4 * H, attn, 1 / math.sqrt(Dh), True,
                        descs=(q_desc, k_desc, k_desc, o_desc)) == N.SUCCESS
    y = dx.clone()
    linear(attn, "o", y, beta=1.0)                 # y = x + attn W_o^T + b_o
    h2 = torch.empty_like(y)
    assert dh.layernorm(y, dg2, dbe2, 1e-5, h2) == N.SUCCESS
    u = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
    linear(h2, "up", u, act=N.ACT_GELU_TANH)       # fused bias + GELU
    out = y.clone()
    linear(u, "down", out, beta=1.0)               # out = y + u W_down^T + b_down
    torch.cuda.synchronize()
    assert bh.execution_status() == N.SUCCESS and dh.execution_status() == N.SUCCESS

    # ---- fp64 CPU chain, rounding to bf16 where the GPU stores bf16
    def lin(a, n, act=None):
        r = a.astype(np.float64) @ w[n].T.astype(np.float64) + b[n]
        return r if act is None else oracle.gelu(r.astype(np.float32), 1)
    r_h1 = bf(oracle.layernorm(x, g1, be1, 1e-5)[0])
    r_qkv = bf(lin(r_h1, "qkv"))
    q = r_qkv[:, :H].reshape(Bt, S, heads, Dh).transpose(0, 2, 1, 3).reshape(Bt * heads, S, Dh)
    k = r_qkv[:, H:2 * H].reshape(Bt, S, heads, Dh).transpose(0, 2, 1, 3).reshape(Bt * heads, S, Dh)
    v = r_qkv[:, 2 * H:].reshape(Bt, S, heads, Dh).transpose(0, 2, 1, 3).reshape(Bt * heads, S, Dh)
    ro, _ = oracle.attention(q, k, v, 1 / math.sqrt(Dh), True)
    r_attn = bf(ro.reshape(Bt, heads, S, Dh).transpose(0, 2, 1, 3).reshape(T, H))
    r_y = bf(x.astype(np.float64) + lin(r_attn, "o"))
    r_h2 = bf(oracle.layernorm(r_y, g2, be2, 1e-5)[0])
    r_u = bf(lin(r_h2, "up", act=True))
    r_out = r_y.astype(np.float64) + lin(r_u, "down")

    got = out.float().cpu().numpy()
    err = np.abs(got - r_out)
    assert np.all(err <= 2e-2 + 2e-2 * np.abs(r_out)), f"max err {err.max()}, {int((err > 2e-2 + 2e-2 * np.abs(r_out)).sum())} bad"
    # and the intermediate the residual path carries
    assert np.all(np.abs(y.float().cpu().numpy() - r_y) <= 2e-2 + 2e-2 * np.abs(r_y))
