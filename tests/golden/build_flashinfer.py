"""Build FlashInfer's trtllm-gen MoE launcher (the reference's F-side expert backend) once, for sm_100a, into
tests/golden/_flashinfer/aot/ -- test and benchmark infrastructure, not part of the product.

    FLASHINFER_CUDA_ARCH_LIST=10.0a python tests/golden/build_flashinfer.py

It runs flashinfer's own JIT recipe (nvcc over the C++ sources flashinfer ships, linked against its prebuilt cubin
package) with the work directory and the cubin include links inside tests/golden/_flashinfer (flashinfer_ref.py),
then copies the module where ``flashinfer_ref.configure`` makes flashinfer load it without compiling.  It needs no
GPU; on 8 host cores it takes about 20 minutes.  The output is git-ignored and travels with the checkout.
"""

import os
import pathlib
import shutil
import sys
import time

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))

import flashinfer_ref  # noqa: E402


def main() -> None:
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    ws = flashinfer_ref.PREBUILT / "ws"
    flashinfer_ref.configure(workspace=ws)
    from flashinfer.jit.fused_moe import gen_trtllm_gen_fused_moe_sm100_module

    t0 = time.time()
    spec = gen_trtllm_gen_fused_moe_sm100_module()
    spec.build(verbose=False)
    src = spec.jit_library_path
    dst = flashinfer_ref.PREBUILT / "aot" / flashinfer_ref.MODULE / f"{flashinfer_ref.MODULE}.so"
    dst.parent.mkdir(parents=True, exist_ok=True)
    shutil.copy2(src, dst)
    print(f"built {dst} ({dst.stat().st_size / 1e6:.1f} MB) in {time.time() - t0:.0f} s")


if __name__ == "__main__":
    main()
