"""The reference's dispatch -> routed experts -> combine semantics in numpy -- test infrastructure only.

Follows, for one MoE layer of one A rank (a replica, group = 1):
  * send:    transport/channel.py:335-355 -- every F rank gets the message; this build sends each F rank only
             the tokens with at least one expert it owns (ascending token order) and F answers row by row,
             which changes no value of the combined output (non-local experts contribute exactly 0).
  * experts: srt/managers/scheduler.py:410-412 FusedMoE(x, StandardTopKOutput(w, ids)) on F rank f with the
             local experts [bounds[f], bounds[f+1]) (scheduler.py:206-218):
                 out[t] = sum_{j: ids[t,j] local} w[t,j] * W2_e (silu(W1_e x_t) * W3_e x_t),  e = ids[t, j]
             with MXFP4 weights, MXFP8 activations (mx.py) and SwiGLU = silu(gate) * up (deepseek_v4.py:51-65,
             swiglu_limit clamp when set).  Top-k weights are used as sent (routed scale pre-fused,
             srt/layers/moe/ep_moe/layer.py:29-36).
  * combine: srt/layers/moe/token_dispatcher/asap.py:174-184 -- fp32 sum of the F partials in F order, cast
             to bf16; then the shared-expert add (srt/batch_overlap/operations_strategy.py:106-111).
Rounding points mirror the CUDA path: GEMM2 rows are rounded to bf16 after the top-k weight, the per-token
reply is an fp32 sum of those rows in ascending slot order rounded to bf16.
"""

from __future__ import annotations

import numpy as np

from . import mx


# ---------------------------------------------------------------- routing (A side)
def f_rank_tables(ids: np.ndarray, bounds) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-F-rank compacted rows.  -> (row_of [F, n] int32 (-1: not routed), count [F], pad [F]).

    Token t goes to F rank f iff one of its ids is in [bounds[f], bounds[f+1]) (the contiguous expert split of
    srt/managers/scheduler.py:206-218); rows keep token order.  A rank that gets no token is announced one padding
    row (count 1, pad 1): a doorbell cannot announce 0 tokens (transport/layout.py:92-102)."""
    ids = np.asarray(ids, dtype=np.int64)
    F = len(bounds) - 1
    n = ids.shape[0]
    row_of = np.full((F, n), -1, dtype=np.int32)
    count = np.zeros(F, dtype=np.int32)
    pad = np.zeros(F, dtype=np.int32)
    for f in range(F):
        hit = np.any((ids >= bounds[f]) & (ids < bounds[f + 1]), axis=1)
        rows = np.cumsum(hit) - 1
        row_of[f, hit] = rows[hit]
        c = int(hit.sum())
        count[f], pad[f] = (c, 0) if c else (1, 1)
    return row_of, count, pad


def expert_counts(ids_f: np.ndarray, e0: int, P: int) -> np.ndarray:
    """Pairs (t, j) per local expert, duplicates counted twice (FusedMoE's per-(token, slot) semantics at
    srt/managers/scheduler.py:410-412)."""
    e = np.asarray(ids_f, dtype=np.int64).reshape(-1) - e0
    return np.bincount(e[(e >= 0) & (e < P)], minlength=P).astype(np.int32)


def expert_permutation(ids_f: np.ndarray, e0: int, P: int):
    """Expert-major order of the local pairs, stable by (expert, token, slot); expert segments start on
    128-row boundaries.  -> (pair_pos [n, k] int32 (-1 non-local), mstart [P+1] tiles, counts [P])."""
    ids_f = np.asarray(ids_f, dtype=np.int64)
    n, k = ids_f.shape
    e = ids_f.reshape(-1) - e0
    local = (e >= 0) & (e < P)
    counts = np.bincount(e[local], minlength=P).astype(np.int32)
    tiles = (counts + 127) // 128
    mstart = np.concatenate([[0], np.cumsum(tiles)]).astype(np.int32)
    pos = np.full(n * k, -1, dtype=np.int64)
    q = np.nonzero(local)[0]
    order = np.lexsort((q, e[q]))  # by expert, then pair index (= token, slot)
    qs = q[order]
    es = e[qs]
    first = np.searchsorted(es, es, side="left")
    rank = np.arange(len(qs)) - first
    pos[qs] = mstart[es] * 128 + rank
    return pos.reshape(n, k).astype(np.int32), mstart, counts


# ---------------------------------------------------------------- weights
def w13_device_rows(I: int) -> np.ndarray:
    """Device row r of w13 -> logical row of the stacked [gate; up] matrix (2I rows): blocks of 256 device
    rows hold gate[128b:128b+128] then up[128b:128b+128]."""
    r = np.arange(2 * I)
    b, within = r // 256, r % 256
    return np.where(within < 128, 128 * b + within, I + 128 * b + (within - 128))


def dequant_w13(w13: np.ndarray, w13_sf: np.ndarray, P: int, H: int, I: int):
    """Device w13 [P, 2I, H/2] bytes + atoms -> (gate [P, I, H], up [P, I, H]) fp32."""
    w13 = np.asarray(w13).reshape(P, 2 * I, H // 2)
    atoms = np.asarray(w13_sf).reshape(P, -1)
    rows = w13_device_rows(I)
    gate = np.zeros((P, I, H), np.float32)
    up = np.zeros((P, I, H), np.float32)
    for e in range(P):
        vals = mx.e2m1_decode(mx.unpack_nibbles(w13[e]))  # [2I, H]
        sf = mx.sf_from_kmajor_atoms(atoms[e], 2 * I, H // 32)
        deq = (vals.reshape(2 * I, H // 32, 32) * mx.e8m0_value(sf)[..., None]).reshape(2 * I, H)
        stacked = np.empty_like(deq)
        stacked[rows] = deq
        gate[e], up[e] = stacked[:I], stacked[I:]
    return gate, up


def dequant_w2(w2: np.ndarray, w2_sf: np.ndarray, P: int, H: int, I: int):
    """Device w2 [P, H, I/2] bytes + atoms -> [P, H, I] fp32."""
    w2 = np.asarray(w2).reshape(P, H, I // 2)
    atoms = np.asarray(w2_sf).reshape(P, -1)
    out = np.zeros((P, H, I), np.float32)
    for e in range(P):
        vals = mx.e2m1_decode(mx.unpack_nibbles(w2[e]))
        sf = mx.sf_from_kmajor_atoms(atoms[e], H, I // 32)
        out[e] = (vals.reshape(H, I // 32, 32) * mx.e8m0_value(sf)[..., None]).reshape(H, I)
    return out


def dequant_fp8(w13_codes, w13_scale, w2_codes, w2_scale):
    """FP8 block-scaled experts (checkpoint layout: w13 [P, 2I, H] gate rows then up rows, scales per 128 x 128)
    -> (gate [P, I, H], up [P, I, H], w2 [P, H, I]) fp32."""
    w13 = mx.fp8_block_dequantize(np.asarray(w13_codes), w13_scale)
    I = w13.shape[1] // 2
    return w13[:, :I], w13[:, I:], mx.fp8_block_dequantize(np.asarray(w2_codes), w2_scale)


# ---------------------------------------------------------------- F side
def silu(x):
    return x / (1.0 + np.exp(-x))


def _act_roundtrip(v, act_quant):
    if act_quant == "fp8":
        return mx.fp8_act_roundtrip(v)
    return mx.mx_roundtrip(v) if act_quant else v


def ffn_pairs(x_f, ids_f, w_f, gate, up, w2, e0: int, P: int, *, act_quant=True, swiglu_limit=None, experts=None):
    """The weighted expert output of every local (token, slot) pair of one message, before the per-token sum:
    -> (y2 [n, k, H] bf16 values as fp32, used [n, k] bool).  One pair = one term of the FusedMoE call of
    srt/managers/scheduler.py:410-412, w[t,j] * W2_e (silu(W1_e x_t) * W3_e x_t) with SwiGLU as
    srt/models/deepseek_v4.py:51-65, rounded to bf16 as the CUDA path stores it.

    x_f: bf16 values (fp32 array) [n_f, H]; ids_f/w_f: [n_f, k]; gate/up [P, I, H]; w2 [P, H, I] (or, with
    ``experts`` = an iterable of local expert indices, only those experts are evaluated and gate/up/w2 are
    indexed by position in that iterable).  act_quant: True = MXFP8 (E8M0 scale per 32) activations, "fp8" = E4M3
    with an fp32 scale per 1 x 128, False = none."""
    x_f = np.asarray(x_f, np.float32)
    ids_f = np.asarray(ids_f, np.int64)
    w_f = np.asarray(w_f, np.float32)
    n, k = ids_f.shape
    H = x_f.shape[1]
    y2 = np.zeros((n, k, H), np.float32)
    used = np.zeros((n, k), bool)
    which = range(P) if experts is None else experts
    for slot, e in enumerate(which):
        tt, jj = np.nonzero(ids_f == e0 + e)
        if tt.size == 0:
            continue
        wi = e if experts is None else slot
        xa = _act_roundtrip(x_f[tt], act_quant)
        g = xa @ gate[wi].T
        u = xa @ up[wi].T
        if swiglu_limit:
            g = np.minimum(g, swiglu_limit)
            u = np.clip(u, -swiglu_limit, swiglu_limit)
        h = _act_roundtrip((silu(g) * u).astype(np.float32), act_quant)
        y = h @ w2[wi].T
        y2[tt, jj] = mx.bf16_round(y * w_f[tt, jj][:, None])
        used[tt, jj] = True
    return y2, used


def reduce_pairs(y2, used):
    """Per-token reply row from its pairs' rows: fp32 sum in ascending slot order, rounded to bf16 (the F
    rank's partial sum that server.py:340-350 sends back; the order is the CUDA reduce's)."""
    y2 = np.asarray(y2, np.float32)
    out = np.zeros((y2.shape[0], y2.shape[2]), np.float32)
    for j in range(y2.shape[1]):
        out += np.where(np.asarray(used)[:, j, None], y2[:, j], 0.0)
    return mx.bf16_round(out)


def ffn_rank(x_f, ids_f, w_f, gate, up, w2, e0: int, P: int, *, act_quant=True, swiglu_limit=None):
    """One F rank's reply for one message: bf16 values as fp32 [n_f, H] -- the FusedMoE call of
    srt/managers/scheduler.py:410-412 over the rank's local experts (``ffn_pairs`` then ``reduce_pairs``)."""
    return reduce_pairs(*ffn_pairs(x_f, ids_f, w_f, gate, up, w2, e0, P, act_quant=act_quant,
                                   swiglu_limit=swiglu_limit))


def combine(parts, row_of, n: int, shared=None):
    """parts[f]: F rank f's reply rows [n_f, H] (bf16 values); row_of [F, n].  -> bf16 values [n, H]: the fp32
    sum over F ranks in F order cast to bf16 (srt/layers/moe/token_dispatcher/asap.py:174-184), then the
    shared-expert add (srt/batch_overlap/operations_strategy.py:106-111)."""
    H = parts[0].shape[1]
    acc = np.zeros((n, H), np.float32)
    for f, part in enumerate(parts):
        rows = row_of[f]
        hit = rows >= 0
        acc[hit] += part[rows[hit]]
    out = mx.bf16_round(acc)
    if shared is not None:
        out = mx.bf16_round(out + np.asarray(shared, np.float32))
    return out


def round_trip(x, ids, w, bounds, experts, *, shared=None, act_quant=True, swiglu_limit=None):
    """A->F->A for one layer.  experts[f] = (gate, up, w2) of F rank f, its experts [bounds[f], bounds[f+1])."""
    x = np.asarray(x, np.float32)
    ids = np.asarray(ids, np.int64)
    w = np.asarray(w, np.float32)
    n = x.shape[0]
    row_of, count, pad = f_rank_tables(ids, bounds)
    parts = []
    for f in range(len(bounds) - 1):
        sel = row_of[f] >= 0
        gate, up, w2 = experts[f]
        P = bounds[f + 1] - bounds[f]
        if sel.any():
            parts.append(ffn_rank(x[sel], ids[sel], w[sel], gate, up, w2, bounds[f], P,
                                  act_quant=act_quant, swiglu_limit=swiglu_limit))
        else:
            parts.append(np.zeros((1, x.shape[1]), np.float32))
    return combine(parts, row_of, n, shared)


# ---------------------------------------------------------------- inputs
def topk_routing(logits: np.ndarray, k: int, kind: str):
    """-> (ids [n, k] int32, weights [n, k] fp32).  'softmax': softmax then top-k renormalised;
    'sigmoid': sigmoid scores, top-k, normalised to sum 1 (DeepSeek-V3 style, no bias)."""
    logits = np.asarray(logits, np.float64)
    if kind == "softmax":
        s = np.exp(logits - logits.max(axis=1, keepdims=True))
        s /= s.sum(axis=1, keepdims=True)
    elif kind == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-logits))
    else:
        raise ValueError(kind)
    ids = np.argsort(-s, axis=1, kind="stable")[:, :k]
    wt = np.take_along_axis(s, ids, axis=1)
    wt = wt / wt.sum(axis=1, keepdims=True)
    return ids.astype(np.int32), wt.astype(np.float32)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
