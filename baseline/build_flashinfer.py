"""Native FlashInfer FA2, the reference's own attention kernel (unpatched), built for sm_100a.

The reference runs FlashInfer's FA2 batch-prefill kernel (`flashinfer-python==0.6.18`, pinned at
final/cooperative_4gpu/code/peer/flashinfer_peer.py:110) for both decode (`use_tensor_cores=True`,
peer/backend.py:130) and append, and uses the unpatched library on gathered all-local KV as its
GPU-side oracle (peer/decode_oracle.py:9-24, peer/cascade_oracle.py:9-28).  This script JIT-builds
that module from the installed FlashInfer (0.6.11.post2 in this image) into
baseline/flashinfer_jit/ (git-ignored; it travels to the GPU box with the built libraries), so the
GPU parity tests and bench.py's native-FlashInfer timing load it instead of compiling on the box.
It is a comparison baseline only: nothing in dual_b200 calls it.

    python baseline/build_flashinfer.py
"""
import os
import pathlib

CACHE = pathlib.Path(__file__).resolve().parent / "flashinfer_jit"


def configure() -> None:
    """Point FlashInfer's JIT cache at baseline/flashinfer_jit (call before `import flashinfer`)."""
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(CACHE))
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")


def build() -> None:
    configure()
    import torch
    from flashinfer.jit.attention.modules import gen_batch_prefill_module

    # the module BatchDecode(use_tensor_cores=True) and BatchPrefill(backend="fa2") load for
    # bf16 q/kv/out, int32 indices, head_dim 128, no RoPE, no sliding window, no soft cap
    gen_batch_prefill_module("fa2", torch.bfloat16, torch.bfloat16, torch.bfloat16, torch.int32, 128, 128, 0,
                             False, False, False).build_and_load()


if __name__ == "__main__":
    build()
    print(f"built native FlashInfer FA2 into {CACHE}")
