"""F-rank expert chain (libasap asap_ffn_job) against the oracle, stage by stage: expert counts and the
expert-major permutation bit-exact, MXFP8 activation codes and scales bit-exact, GEMM1 (SwiGLU + requant) and
GEMM2 (top-k weighted) within relative L2 1e-2 of the oracle evaluated on the kernel's own quantised inputs, and
the reply rows within relative L2 1e-2 of the reference semantics with the same activation quantisation."""

import numpy as np
import pytest
import torch

from asap_b200.experts import Mxfp4Experts
from asap_b200.quant import mxfp4_quantize
from gpu_util import FfnHarness, bf16_tensor_from_np, device_bytes, experts_to_oracle, np_from_bf16, random_inputs
from oracle import moe, mx

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative L2


def check_chain(h: FfnHarness, x, ids, w, gate, up, w2, e0, P, swiglu_limit=None):
    n, k = ids.shape
    H, I = h.e.hidden, h.e.inter
    # counts and permutation: bit-exact
    pos_ref, mstart_ref, counts_ref = moe.expert_permutation(ids, e0, P)
    counts = device_bytes(h.ptrs["ecnt"], 4 * P).view(np.int32)
    np.testing.assert_array_equal(counts, counts_ref)
    pos = device_bytes(h.ptrs["pair_pos"], 4 * n * k).view(np.int32).reshape(n, k)
    np.testing.assert_array_equal(pos, pos_ref)
    rows = int(mstart_ref[-1]) * 128
    tt, jj = np.nonzero(pos_ref >= 0)
    prow = pos_ref[tt, jj]
    # activation quantisation: bit-exact (expert-major rows and scale atoms)
    xq = device_bytes(h.ptrs["xq"], rows * H).reshape(rows, H)
    xsf = mx.sf_from_atoms(device_bytes(h.ptrs["xq_sf"], rows * H // 32), rows, H // 32)
    q_ref, s_ref = mx.mx_quantize(x[tt])
    np.testing.assert_array_equal(xq[prow], q_ref)
    np.testing.assert_array_equal(xsf[prow], s_ref)
    # GEMM1 + SwiGLU + requant, against the oracle on the same quantised activations
    xa = mx.mx_dequantize(xq[prow], xsf[prow])
    e_of = ids[tt, jj] - e0
    g = np.zeros((len(prow), I), np.float32)
    u = np.zeros((len(prow), I), np.float32)
    for ex in range(P):  # per expert: never materialise weights per pair
        sel = e_of == ex
        if sel.any():
            g[sel] = xa[sel] @ gate[ex].T
            u[sel] = xa[sel] @ up[ex].T
    if swiglu_limit:
        g = np.minimum(g, swiglu_limit)
        u = np.clip(u, -swiglu_limit, swiglu_limit)
    h_ref = (moe.silu(g) * u).astype(np.float32)
    hq = device_bytes(h.ptrs["hq"], rows * I).reshape(rows, I)
    hsf = mx.sf_from_atoms(device_bytes(h.ptrs["hq_sf"], rows * I // 32), rows, I // 32)
    h_gpu = mx.mx_dequantize(hq[prow], hsf[prow])
    # the kernel stores h in MXFP8: compare with the oracle's MXFP8 rounding of its own h
    hq_ref, hsf_ref = mx.mx_quantize(h_ref)
    assert moe.rel_l2(h_gpu, mx.mx_dequantize(hq_ref, hsf_ref)) < TOL
    assert np.mean(hq[prow] == hq_ref) > 0.9  # codes differ only where fp32 accumulation order tips a rounding
    assert moe.rel_l2(h_gpu, h_ref) < 6e-2     # the MXFP8 rounding itself (3 mantissa bits)
    # GEMM2 + top-k weight, on the kernel's own h
    y_ref = np.zeros((len(prow), H), np.float32)
    for ex in range(P):
        sel = e_of == ex
        if sel.any():
            y_ref[sel] = h_gpu[sel] @ w2[ex].T
    y_ref *= w[tt, jj][:, None]
    y2 = device_bytes(h.ptrs["y2"], rows * H * 2).view(np.uint16).reshape(rows, H)
    y_gpu = mx.bf16_from_bits(y2[prow])
    assert moe.rel_l2(y_gpu, y_ref) < TOL
    # reply rows: reference semantics with the same activation quantisation
    out_ref = moe.ffn_rank(x, ids, w, gate, up, w2, e0, P, act_quant=True, swiglu_limit=swiglu_limit)
    out = np_from_bf16(h.reply[:n])
    assert moe.rel_l2(out, out_ref) < TOL
    return out, out_ref


@pytest.mark.parametrize("n,k,P,H,I,e0", [
    (64, 2, 4, 256, 128, 4),       # one tile each way, non-zero expert base
    (300, 4, 6, 512, 256, 0),      # several experts > 128 rows, two n-tiles in GEMM1/GEMM2
    (64, 12, 16, 256, 128, 0),     # more than 8 local experts per token (the reduce's long path)
    (8192, 8, 256, 256, 128, 0),   # the maximum of 256 local experts, 128 permutation chunks (config 2's routing)
])
def test_ffn_chain_random_weights(cuda_ok, n, k, P, H, I, e0):
    rng = np.random.default_rng(n)
    e = Mxfp4Experts.random(P, H, I, expert_base=e0, seed=n)
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, e0 - 2, e0 + P + 2, bias_expert=e0)  # some ids are not local
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), seq=41)
    check_chain(h, x, ids, w, gate, up, w2, e0, P)
    assert int(h.done[0].item()) == 41
    h.release()
    e.release()


def test_ffn_chain_config1_weights(cuda_ok):
    """Benchmark config 1's F rank 1 (experts 8..15 of 16, H=1024, I=512, top-2 softmax, T=512): fp32 weights
    N(0, 0.02) quantised to MXFP4 on the host, through the logical -> device layout packer."""
    rng = np.random.default_rng(0)
    T, H, I, E, k = 512, 1024, 512, 16, 2
    e0, P = 8, 8
    w13 = rng.standard_normal((P, 2 * I, H)).astype(np.float32) * 0.02
    w2f = rng.standard_normal((P, H, I)).astype(np.float32) * 0.02
    c13, s13 = mxfp4_quantize(w13)
    c2, s2 = mxfp4_quantize(w2f)
    e = Mxfp4Experts.from_logical(c13, s13, c2, s2, expert_base=e0)
    deq13 = mx.e2m1_decode(c13).reshape(P, 2 * I, H // 32, 32) * mx.e8m0_value(s13)[..., None]
    deq13 = deq13.reshape(P, 2 * I, H)
    gate, up = deq13[:, :I], deq13[:, I:]
    w2 = (mx.e2m1_decode(c2).reshape(P, H, I // 32, 32) * mx.e8m0_value(s2)[..., None]).reshape(P, H, I)
    x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((T, E)), k, "softmax")
    h = FfnHarness(e, n_max=T, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    out, out_ref = check_chain(h, x, ids, w, gate, up, w2, e0, P)
    # against the bf16 result of the same dequantised weights without activation quantisation (reported bound)
    plain = moe.ffn_rank(x, ids, w, gate, up, w2, e0, P, act_quant=False)
    assert moe.rel_l2(out, plain) < 8e-2
    h.release()
    e.release()


def test_ffn_chain_swiglu_limit(cuda_ok):
    rng = np.random.default_rng(3)
    n, k, P, H, I = 128, 2, 4, 256, 128
    e = Mxfp4Experts.random(P, H, I, seed=3, scale_lo=121, scale_hi=123)  # large activations: the clamp bites
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, 0, P)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), swiglu_limit=2.0)
    check_chain(h, x, ids, w, gate, up, w2, 0, P, swiglu_limit=2.0)
    h.release()
    e.release()


def test_ffn_chain_no_local_pair(cuda_ok):
    """A padding row (ids -1, what dispatch sends an F rank that got no token): the reply row is exactly 0."""
    e = Mxfp4Experts.random(4, 256, 128, seed=9)
    h = FfnHarness(e, n_max=4, topk=2)
    h.reply.fill_(1.0)
    x = torch.randn(1, 256, device="cuda").to(torch.bfloat16)
    ids = torch.full((1, 2), -1, dtype=torch.int32, device="cuda")
    w = torch.zeros(1, 2, device="cuda")
    h.run(x, ids, w, seq=5)
    assert torch.count_nonzero(h.reply[0]).item() == 0
    assert int(h.done[0].item()) == 5
    h.release()
    e.release()


def test_ffn_chain_deepseek_dims(cuda_ok):
    """DeepSeek-V3 expert shape (H=7168, I=2048: 56 K-tiles in GEMM1, 16 N-tiles / 28 N-tiles) on 8 experts."""
    rng = np.random.default_rng(11)
    n, k, P, H, I = 256, 8, 8, 7168, 2048
    e = Mxfp4Experts.random(P, H, I, seed=11, scale_lo=117, scale_hi=120)
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, 0, 12)  # 8 of 12 experts local
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    check_chain(h, x, ids, w, gate, up, w2, 0, P)
    h.release()
    e.release()


@pytest.mark.parametrize("n,k,P,H,I,e0", [
    (64, 2, 4, 256, 128, 4),        # every expert in one block of <= 64 rows
    (300, 4, 6, 512, 256, 0),       # experts over 128 rows: full blocks and a tail block
    (64, 12, 16, 256, 128, 0),      # more than 8 local experts per token
    (40, 8, 32, 1024, 512, 0),      # config-5-like: many experts, a handful of rows each (mostly padding blocks)
])
def test_ffn_chain_small_segments(cuda_ok, n, k, P, H, I, e0):
    """Small jobs (few rows per expert, most of each 128-row block padding): the bit-exact routing / activation
    codes and the tolerances of the other chain tests."""
    rng = np.random.default_rng(n + 1000)
    e = Mxfp4Experts.random(P, H, I, expert_base=e0, seed=n + 3)
    gate, up, w2 = experts_to_oracle(e)
    x, ids, w = random_inputs(rng, n, H, k, e0 - 2, e0 + P + 2, bias_expert=e0)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), seq=23)
    check_chain(h, x, ids, w, gate, up, w2, e0, P)
    assert int(h.done[0].item()) == 23
    h.release()
    e.release()


def test_ffn_chain_duplicate_ids_and_limits(cuda_ok):
    """Edge cases of the routing input: duplicate expert ids within one token's top-k (each pair counts, as
    FusedMoE sums them), the largest top-k (32) and the largest local expert count (256), a message of exactly n_max
    tokens, ids outside the local range."""
    rng = np.random.default_rng(31)
    n, k, P, H, I = 96, 32, 256, 256, 128
    e = Mxfp4Experts.random(P, H, I, seed=12)
    gate, up, w2 = experts_to_oracle(e)
    ids = rng.integers(-3, P + 3, (n, k)).astype(np.int32)  # duplicates and non-local ids on purpose
    ids[:10, 1] = ids[:10, 0]
    w = rng.random((n, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), seq=5)
    check_chain(h, x, ids, w, gate, up, w2, 0, P)
    assert int(h.done[0].item()) == 5
    h.release()
    e.release()


def test_ffn_chain_from_checkpoint(cuda_ok, tmp_path):
    """F-rank weight ingest end to end: a safetensors shard with two ranks' experts over two layers (DeepSeek-V4
    names, int8 codes and float8_e8m0fnu scales mixed in); `ingest.load_layer` reads this rank's experts of one
    layer, the registered bytes dequantise to the checkpoint's weights, and the chain matches the oracle."""
    from safetensors.torch import save_file

    from asap_b200 import ingest

    rng = np.random.default_rng(8)
    H, I, layer = 256, 128, 1
    mine, others = range(4, 8), range(0, 4)
    tensors, logical = {}, {}
    for l in (0, 1):
        for e in list(others) + list(mine):
            for p, name, (rows, kk) in (("gate", "w1", (I, H)), ("up", "w3", (I, H)), ("down", "w2", (H, I))):
                codes = rng.integers(0, 16, (rows, kk)).astype(np.uint8)
                scales = rng.integers(117, 121, (rows, kk // 32)).astype(np.uint8)
                w = torch.from_numpy(mx.pack_nibbles(codes))
                s = torch.from_numpy(scales)
                if e % 2:
                    w = w.view(torch.int8)
                if e % 3 == 0 and hasattr(torch, "float8_e8m0fnu"):
                    s = s.view(torch.float8_e8m0fnu)
                tensors[f"layers.{l}.ffn.experts.{e}.{name}.weight"] = w
                tensors[f"layers.{l}.ffn.experts.{e}.{name}.scale"] = s
                logical[l, e, p] = mx.e2m1_decode(codes) * np.repeat(mx.e8m0_value(scales), 32, axis=-1)
    tensors["layers.1.ffn.shared_experts.w1.weight"] = torch.zeros(4, 4)
    path = str(tmp_path / "model-00001.safetensors")
    save_file(tensors, path)
    e = ingest.load_layer([path], layer, mine, num_layers=2)
    assert (e.num_local, e.expert_base, e.hidden, e.inter) == (4, 4, H, I)
    gate, up, w2 = experts_to_oracle(e)
    for i, ex in enumerate(mine):
        np.testing.assert_array_equal(gate[i], logical[layer, ex, "gate"])
        np.testing.assert_array_equal(up[i], logical[layer, ex, "up"])
        np.testing.assert_array_equal(w2[i], logical[layer, ex, "down"])
    n, k = 200, 4
    x, ids, w = random_inputs(rng, n, H, k, 2, 10, bias_expert=4)
    h = FfnHarness(e, n_max=n, topk=k)
    h.run(bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    check_chain(h, x, ids, w, gate, up, w2, 4, 4)
    h.release()
    e.release()
