"""The reference-facing C++ layer (mini-lla_b200/host): mini-lla's own
GPU operator API served by libmlb.so.

- CPU: the reference's unchanged src/cuda_forward.cc, compiled against the
  reference headers, needs exactly the cuda_ops.h symbols this layer's
  cuda_ops.cc defines (link surface of the drop-in).
- GPU: oracle/_ref/mlb_dropin_test runs the reference API (CudaRmsNorm,
  CudaRope, CudaEmbeddingRow, ... and the row-batched additions) against the
  reference's CPU operators.
Both binaries are built by `make -C oracle dropin` where the reference
headers are present; the tests skip when they were not built.
"""
import os
import subprocess

import pytest

from conftest import ORACLE_DIR

REF = os.path.join(ORACLE_DIR, "_ref")


def test_cuda_forward_links_against_this_layer():
    fwd = os.path.join(REF, "cuda_forward.o")
    ops = os.path.join(REF, "cuda_ops_host.o")
    if not all(os.path.exists(p) for p in
               (fwd, ops, os.path.join(REF, "cuda_matmul_host.o"),
                os.path.join(REF, "cuda_attention_host.o"))):
        pytest.skip("drop-in objects not built (reference headers absent)")
    undefined = subprocess.run(["nm", "-C", "--undefined-only", fwd], check=True,
                               capture_output=True, text=True).stdout
    needed = {l.split("U ", 1)[1].strip() for l in undefined.splitlines()
              if "U mini_lla::Cuda" in l}
    have = set()
    for obj in (ops, os.path.join(REF, "cuda_matmul_host.o"),
                os.path.join(REF, "cuda_attention_host.o")):
        defined = subprocess.run(["nm", "-C", "--defined-only", obj], check=True,
                                 capture_output=True, text=True).stdout
        have |= {l.split(" ", 2)[2].strip() for l in defined.splitlines()
                 if " T mini_lla::Cuda" in l}
    # the operator entry points cuda_forward.cc calls (cuda_ops.h:11-34), its
    # linear layer (cuda_matmul.h:11) and its KV cache + attention
    # (cuda_attention.h:8-45)
    ops_needed = {n for n in needed if n.split("(")[0] in {
        "mini_lla::CudaRmsNorm", "mini_lla::CudaRope", "mini_lla::CudaSilu",
        "mini_lla::CudaMul", "mini_lla::CudaAdd", "mini_lla::CudaSoftmax",
        "mini_lla::CudaEmbeddingRow", "mini_lla::CudaAddBias",
        "mini_lla::CudaLinear", "mini_lla::CudaAttention",
        "mini_lla::CudaKvCache::Write", "mini_lla::CudaKvCache::Reset"}}
    assert len(ops_needed) >= 10, needed
    missing = ops_needed - have
    assert not missing, f"cuda_ops.cc lacks {missing}"


@pytest.mark.gpu
def test_reference_api_dropin_binary():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = os.path.join(REF, "mlb_dropin_test")
    if not os.path.exists(exe):
        pytest.skip("mlb_dropin_test not built (reference headers absent)")
    res = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "dropin ok" in res.stdout


@pytest.mark.gpu
def test_prefill_driver_and_weight_upload_binary():
    """oracle/_ref/mlb_forward_test: ForwardBatchCuda (row-batched prefill)
    and the device weight / GGUF upload paths against the reference's CPU
    ForwardBatch and its per-token GPU driver on random models (Q8_0, Q4_0,
    Q4_1, F32; GQA, biases, NeoX, tied output) and on the reference's GGUF
    test fixture; logits within 2e-5 of the largest logit."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = os.path.join(REF, "mlb_forward_test")
    if not os.path.exists(exe):
        pytest.skip("mlb_forward_test not built (reference headers absent)")
    res = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "forward ok" in res.stdout


def test_device_list_parsing_and_validation():
    """oracle/_ref/mlb_devices_test --cpu: the multi-device backend's device
    lists ("all", "0,2,3") and their validation with the reference's
    exception types (backend.cc:26-42: invalid_argument for devices on a CPU
    backend, out_of_range for an id outside the visible count; duplicates and
    empty lists rejected), run against a given device count without a GPU."""
    exe = os.path.join(REF, "mlb_devices_test")
    if not os.path.exists(exe):
        pytest.skip("mlb_devices_test not built (reference headers absent)")
    res = subprocess.run([exe, "--cpu"], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "devices cpu ok" in res.stdout


@pytest.mark.gpu
def test_layer_ops_and_requests_split_across_devices():
    """oracle/_ref/mlb_devices_test on two or more GPUs: weights replicated
    from a host model and from the reference's GGUF fixture (every replica
    byte-identical, on its own device); the layer-op chain over 1001 token
    rows split across devices 0,1 and 1,0 bit-identical to one device, with
    device 1's own RoPE table and pool; five requests spread over two devices
    by ForwardBatchesCuda (prefill, then a decode step) bit-identical to one
    device; a context moved to another device refused."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    exe = os.path.join(REF, "mlb_devices_test")
    if not os.path.exists(exe):
        pytest.skip("mlb_devices_test not built (reference headers absent)")
    res = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "devices ok" in res.stdout
