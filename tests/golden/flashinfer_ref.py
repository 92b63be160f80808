"""FlashInfer's trtllm-gen MXFP4 MoE -- the expert backend the reference's F ranks run -- as a parity source and a
timing bar.  TEST AND BENCHMARK INFRASTRUCTURE ONLY: the product path never imports it.

The reference's F rank runs SGLang FusedMoE on ``--moe-runner-backend flashinfer_mxfp4`` (scripts/run_asap.sh:99),
which calls ``flashinfer.fused_moe.trtllm_fp4_block_scale_routed_moe`` with MXFP8 activations and MXFP4 weights
(python/sgl_asap_plugin/srt/layers/quantization/mxfp4_flashinfer_trtllm_moe.py:68-99).  Here that function is
called the same way on this GPU's memory only: its kernels are run and timed, never inspected.

Weight layout the kernels read (built from checkpoint-order tensors with flashinfer's own Python helpers):
  * W13 rows in [up (W3); gate (W1)] order, interleaved up/gate per row pair and shuffled in blocks of 32 rows for
    an epilogue tile of 128 (``_maybe_get_cached_w3_w1_permute_indices``); W2 rows shuffled the same way
    (``get_w2_permute_indices_with_cache``);
  * E8M0 scales permuted with their rows, then in the 128 x 4 swizzled layout: byte c % 4 + (c / 4) * 512 +
    (r % 32) * 16 + ((r % 128) / 32) * 4 + (r / 128) * 128 * cols for row r, 32-block c (the published layout of
    flashinfer's ``compute_sf_index_swizzled_128x4``; written here in torch, so no second JIT module is built);
  * activations: E4M3 codes [T, H] with E8M0 scales [T, H / 32] in linear layout;
  * routing: int32 per (token, slot), expert id in the high 16 bits and the bf16 bits of its weight in the low 16
    (the packing flashinfer's autotuner builds for this op), so the routing weights are bf16-rounded.

The compiled launcher is a JIT module of flashinfer (C++ sources shipped with it, linked against its prebuilt
cubins).  ``tests/golden/build_flashinfer.py`` builds it once into ``tests/golden/_flashinfer/aot`` (git-ignored,
shipped to the GPU machine with the checkout); ``configure()`` points flashinfer at that build and at a cubin directory
under ``tests/golden/_flashinfer/cubins`` whose entries link to the installed cubin package, so flashinfer's
header links are made inside the checkout and nothing is compiled or written elsewhere at run time.
"""

from __future__ import annotations

import os
import pathlib

import torch

HERE = pathlib.Path(__file__).resolve().parent
PREBUILT = HERE / "_flashinfer"
MODULE = "fused_moe_trtllm_sm100"


def _mirror_cubins(real: pathlib.Path, mirror: pathlib.Path) -> None:
    """Make ``mirror`` a directory whose entries link to those of the installed cubin package (except the
    generated include tree flashinfer links there itself)."""
    mirror.mkdir(parents=True, exist_ok=True)
    for entry in os.listdir(real):
        if entry == "flashinfer":
            continue
        link = mirror / entry
        if not link.exists():
            os.symlink(real / entry, link)


def configure(workspace: pathlib.Path | None = None):
    """Point flashinfer's JIT at the in-checkout cubin mirror and prebuilt module directory (call before the MoE
    module is first used).  -> the flashinfer.fused_moe.core module."""
    import flashinfer.jit.cubin_loader as cubin_loader
    import flashinfer.jit.env as jit_env

    real = pathlib.Path(jit_env.FLASHINFER_CUBIN_DIR)
    mirror = PREBUILT / "cubins"
    if real.resolve() != mirror.resolve():
        _mirror_cubins(real, mirror)
        jit_env.FLASHINFER_CUBIN_DIR = mirror
        cubin_loader.FLASHINFER_CUBIN_DIR = mirror
    jit_env.FLASHINFER_AOT_DIR = PREBUILT / "aot"
    if workspace is not None:
        jit_env.FLASHINFER_JIT_DIR = workspace / "cached_ops"
        jit_env.FLASHINFER_WORKSPACE_DIR = workspace
    from flashinfer.fused_moe import core

    return core


def available() -> str | None:
    """None when the prebuilt module is present, else why not."""
    so = PREBUILT / "aot" / MODULE / f"{MODULE}.so"
    if not so.exists():
        return f"flashinfer MoE module not built ({so} missing; run tests/golden/build_flashinfer.py)"
    try:
        import flashinfer  # noqa: F401
    except Exception as exc:  # noqa: BLE001
        return f"flashinfer does not import: {type(exc).__name__}: {exc}"
    return None


def swizzle_128x4(sf: torch.Tensor) -> torch.Tensor:
    """[rows, cols] scale bytes (rows % 128 == 0, cols % 4 == 0) -> the 128 x 4 swizzled bytes, flat."""
    rows, cols = sf.shape
    r = torch.arange(rows, device=sf.device).view(rows, 1)
    c = torch.arange(cols, device=sf.device).view(1, cols)
    off = c % 4 + (c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (r // 128) * (128 * cols)
    out = torch.empty(rows * cols, dtype=torch.uint8, device=sf.device)
    out[off.reshape(-1)] = sf.reshape(-1)
    return out


def weights_for_kernel(w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor):
    """Checkpoint-order MXFP4 experts (w13 [P, 2I, H/2] rows gate then up, s13 [P, 2I, H/32] E8M0 bytes,
    w2 [P, H, I/2], s2 [P, H, I/32]; CUDA uint8) -> (w13, s13, w2, s2) as the trtllm-gen kernels read them."""
    core = configure()
    P, two_i, _ = w13.shape
    inter = two_i // 2
    w31 = torch.cat([w13[:, inter:], w13[:, :inter]], dim=1)  # [up; gate]
    s31 = torch.cat([s13[:, inter:], s13[:, :inter]], dim=1)
    cache = {}
    out13, sf13, out2, sf2 = [], [], [], []
    for e in range(P):
        rows = core._maybe_get_cached_w3_w1_permute_indices(cache, w31[e], 128).to(w13.device)
        out13.append(w31[e][rows].contiguous())
        rows_sf = core._maybe_get_cached_w3_w1_permute_indices(cache, s31[e], 128, num_elts_per_sf=32).to(w13.device)
        sf13.append(swizzle_128x4(s31[e][rows_sf].contiguous()))
        rows2 = core.get_w2_permute_indices_with_cache(cache, w2[e], 128).to(w2.device)
        out2.append(w2[e][rows2].contiguous())
        rows2_sf = core.get_w2_permute_indices_with_cache(cache, s2[e], 128, num_elts_per_sf=32).to(w2.device)
        sf2.append(swizzle_128x4(s2[e][rows2_sf].contiguous()))
    f8 = torch.float8_e4m3fn
    return (torch.stack(out13), torch.stack(sf13).view(f8).reshape(P, two_i, -1), torch.stack(out2),
            torch.stack(sf2).view(f8).reshape(P, w2.shape[1], -1))


def mxfp8_quantize(x: torch.Tensor):
    """bf16/fp32 [T, H] on the GPU -> (E4M3 codes [T, H] as torch.float8_e4m3fn, E8M0 bytes [T, H/32]) by the OCP
    Microscaling v1.0 rule (scale 2^(floor(log2 amax) - 8), elements rounded to nearest even, saturated at 448)."""
    v = x.float().reshape(x.shape[0], -1, 32)
    amax = v.abs().amax(dim=-1)
    s = torch.clamp(((amax.view(torch.int32) >> 23) & 0xFF) - 8, min=0)
    inv = torch.ldexp(torch.ones_like(amax), (127 - s).float())
    q = (v * inv[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), s.to(torch.uint8)


def pack_routing(ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Top-k ids and weights -> the packed int32 routing words (id << 16 | bf16 bits of the weight)."""
    bits = w.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return (ids.to(torch.int32) << 16) | bits


def random_weights(P: int, hidden: int, inter: int, seed: int, device="cuda"):
    """Uniform random E2M1 codes and E8M0 scales 2^-10..2^-7 (the benchmark's synthetic experts), checkpoint order,
    laid out for the kernels."""
    g = torch.Generator(device=device).manual_seed(seed)

    def rnd(shape, lo, hi):
        return torch.randint(lo, hi + 1, shape, dtype=torch.uint8, device=device, generator=g)

    return weights_for_kernel(rnd((P, 2 * inter, hidden // 2), 0, 255), rnd((P, 2 * inter, hidden // 32), 117, 120),
                              rnd((P, hidden, inter // 2), 0, 255), rnd((P, hidden, inter // 32), 117, 120))


def run(xq: torch.Tensor, xsf: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, weights, num_experts: int,
        intermediate: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """One MoE call: xq E4M3 [T, H] (torch.float8_e4m3fn), xsf E8M0 bytes [T, H/32] (uint8), ids/w [T, k] ->
    bf16 [T, H] = sum_j w[t, j] * W2_e swiglu(W13_e x_t) over the experts, as the reference's F rank computes."""
    core = configure()
    w13, s13, w2, s2 = weights
    T, k = ids.shape
    if out is None:
        out = torch.empty(T, xq.shape[1], dtype=torch.bfloat16, device=xq.device)
    from flashinfer.tllm_enums import ActivationType, RoutingMethodType

    core.trtllm_fp4_block_scale_routed_moe(
        topk_ids=pack_routing(ids, w), routing_bias=None, hidden_states=xq,
        hidden_states_scale=xsf.view(torch.float8_e4m3fn).reshape(T, -1), gemm1_weights=w13,
        gemm1_weights_scale=s13, gemm1_bias=None, gemm1_alpha=None, gemm1_beta=None, gemm1_clamp_limit=None,
        gemm2_weights=w2, gemm2_weights_scale=s2, gemm2_bias=None, output1_scale_scalar=None,
        output1_scale_gate_scalar=None, output2_scale_scalar=None, num_experts=num_experts, top_k=k, n_group=None,
        topk_group=None, intermediate_size=intermediate, local_expert_offset=0, local_num_experts=num_experts,
        routed_scaling_factor=None, routing_method_type=int(RoutingMethodType.TopK), do_finalize=True,
        activation_type=ActivationType.Swiglu.value, output=out, tune_max_num_tokens=max(8, 1 << (T - 1).bit_length()))
    return out
