"""F-rank expert chain with FP8 block-scaled experts (E4M3 weights, fp32 scale per 128 x 128 block; E4M3
activations with an fp32 scale per 1 x 128) against the oracle, stage by stage: expert counts and permutation
bit-exact, activation codes and scales bit-exact, GEMM1 (SwiGLU + requant) and GEMM2 (top-k weighted) within
relative L2 1e-2 of the oracle on the kernel's own quantised inputs, reply rows within 1e-2 of the reference
semantics with the same activation quantisation; then the round trip with two FP8 F ranks."""

import numpy as np
import pytest
import torch

from asap_b200.experts import Fp8Experts
from asap_b200.loopback import Loopback
from asap_b200.transport.layout import Geometry
from gpu_util import FfnHarness, bf16_tensor_from_np, device_bytes, experts_to_oracle, np_from_bf16, random_inputs
from oracle import moe, mx

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative L2


def m_cap_of(n_max, topk, P):
    return (n_max * topk + 128 * P + 127) // 128 * 128


def check_chain_fp8(h: FfnHarness, x, ids, w, gate, up, w2, e0, P, swiglu_limit=None):
    n, k = ids.shape
    H, I = h.e.hidden, h.e.inter
    m_cap = m_cap_of(h.n_max, h.topk, P)
    pos_ref, mstart_ref, counts_ref = moe.expert_permutation(ids, e0, P)
    np.testing.assert_array_equal(device_bytes(h.ptrs["ecnt"], 4 * P).view(np.int32), counts_ref)
    pos = device_bytes(h.ptrs["pair_pos"], 4 * n * k).view(np.int32).reshape(n, k)
    np.testing.assert_array_equal(pos, pos_ref)
    rows = int(mstart_ref[-1]) * 128
    tt, jj = np.nonzero(pos_ref >= 0)
    prow = pos_ref[tt, jj]
    # activations: E4M3 rows and fp32 scales (K-block-major [H/128][m_cap]) bit-exact
    xq = device_bytes(h.ptrs["xq"], rows * H).reshape(rows, H)
    xsf = device_bytes(h.ptrs["xq_sf"], 4 * m_cap * (H // 128)).view(np.float32).reshape(H // 128, m_cap).T
    q_ref, s_ref = mx.fp8_act_quantize(x[tt])
    np.testing.assert_array_equal(xq[prow], q_ref)
    np.testing.assert_array_equal(xsf[prow], s_ref)
    # GEMM1 with block-scale promotion + SwiGLU + 1x128 requant, against the oracle on the same inputs
    xa = mx.fp8_act_dequantize(xq[prow], xsf[prow])
    e_of = ids[tt, jj] - e0
    g = np.zeros((len(prow), I), np.float32)
    u = np.zeros((len(prow), I), np.float32)
    for ex in range(P):
        sel = e_of == ex
        if sel.any():
            g[sel] = xa[sel] @ gate[ex].T
            u[sel] = xa[sel] @ up[ex].T
    if swiglu_limit:
        g = np.minimum(g, swiglu_limit)
        u = np.clip(u, -swiglu_limit, swiglu_limit)
    h_ref = (moe.silu(g) * u).astype(np.float32)
    hq = device_bytes(h.ptrs["hq"], rows * I).reshape(rows, I)
    hsf = device_bytes(h.ptrs["hq_sf"], 4 * m_cap * (I // 128)).view(np.float32).reshape(I // 128, m_cap).T
    h_gpu = mx.fp8_act_dequantize(hq[prow], hsf[prow])
    hq_ref, hsf_ref = mx.fp8_act_quantize(h_ref)
    assert moe.rel_l2(h_gpu, mx.fp8_act_dequantize(hq_ref, hsf_ref)) < TOL
    assert np.mean(hq[prow] == hq_ref) > 0.9
    np.testing.assert_allclose(hsf[prow], hsf_ref, rtol=1e-3)
    # GEMM2 + top-k weight, on the kernel's own h
    y_ref = np.zeros((len(prow), H), np.float32)
    for ex in range(P):
        sel = e_of == ex
        if sel.any():
            y_ref[sel] = h_gpu[sel] @ w2[ex].T
    y_ref *= w[tt, jj][:, None]
    y2 = device_bytes(h.ptrs["y2"], rows * H * 2).view(np.uint16).reshape(rows, H)
    assert moe.rel_l2(mx.bf16_from_bits(y2[prow]), y_ref) < TOL
    out_ref = moe.ffn_rank(x, ids, w, gate, up, w2, e0, P, act_quant="fp8", swiglu_limit=swiglu_limit)
    out = np_from_bf16(h.reply[:n])
    assert moe.rel_l2(out, out_ref) < TOL
    return out, out_ref


@pytest.mark.parametrize("n,k,P,H,I,e0", [
    (64, 2, 4, 256, 128, 4),        # one tile each way, non-zero expert base
    (300, 4, 6, 512, 256, 0),       # several experts > 128 rows, two n-tiles in both GEMMs
    (64, 12, 16, 256, 128, 0),      # more than 8 local experts per token
    (1000, 4, 8, 2048, 512, 0),     # 16 K blocks, more tiles than CTAs (the TMEM ping-pong across tiles)
])
def test_fp8_chain_random_weights(cuda_ok, n, k, P, H, I, e0):
    rng = np.random.default_rng(n)
    e = Fp8Experts.random(P, H, I, expert_base=e0, seed=n)
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, e0 - 2, e0 + P + 2, bias_expert=e0)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), seq=17)
    check_chain_fp8(h, x, ids, w, gate, up, w2, e0, P)
    assert int(h.done[0].item()) == 17
    h.release()
    e.release()


def test_fp8_swiglu_limit(cuda_ok):
    rng = np.random.default_rng(5)
    n, k, P, H, I = 128, 2, 4, 256, 256
    e = Fp8Experts.random(P, H, I, seed=9, std=0.2)  # large pre-activations, so the clamp bites
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, 0, P)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), swiglu_limit=1.5)
    check_chain_fp8(h, x, ids, w, gate, up, w2, 0, P, swiglu_limit=1.5)
    h.release()
    e.release()


def test_fp8_config4_layer_shape(cuda_ok):
    """Config 4's expert shape (H=8192, I=3584: 64 K blocks in GEMM1, 28 in GEMM2) on 2 local experts."""
    rng = np.random.default_rng(4)
    n, k, P, H, I = 160, 2, 2, 8192, 3584
    e = Fp8Experts.random(P, H, I, seed=4)
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, 0, P + 2)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    check_chain_fp8(h, x, ids, w, gate, up, w2, 0, P)
    h.release()
    e.release()


def test_fp8_round_trip_two_f_ranks(cuda_ok):
    """Config 4's routing shape scaled down: 16 experts over 2 FP8 F ranks, top-6 softmax, one A replica."""
    rng = np.random.default_rng(6)
    T, H, I, k = 400, 512, 256, 6
    per_f = [{0: Fp8Experts.random(8, H, I, expert_base=8 * f, seed=20 + f)} for f in range(2)]
    lb = Loopback(Geometry(1, 1, 2, T, H, k, 2), per_f, timeout_s=5.0)
    lb.install()
    try:
        from asap_b200.dispatcher import AsapDispatcher
        from asap_b200.sglang_shim import StandardTopKOutput

        ow = [experts_to_oracle(d[0]) for d in per_f]
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        ids, w = moe.topk_routing(rng.standard_normal((T, 16)), k, "softmax")
        shared = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        disp = AsapDispatcher(0)
        d = disp.dispatch(bf16_tensor_from_np(x), StandardTopKOutput(torch.from_numpy(w).cuda(),
                                                                     torch.from_numpy(ids).cuda()))
        out = disp.combine(d, shared=bf16_tensor_from_np(shared))
        torch.cuda.synchronize()
        lb.check()
        ref = moe.round_trip(x, ids, w, [0, 8, 16], ow, shared=shared, act_quant="fp8")
        assert moe.rel_l2(np_from_bf16(out), ref) < TOL
    finally:
        lb.close()
        for dct in per_f:
            dct[0].release()
