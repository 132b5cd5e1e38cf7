"""One process driving two GPUs: launch attributes, tensor maps, error words and launch
caches are per device, so the same linear must run (bit-exact) on a second device after
the first.  Skipped on one-GPU hosts."""

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in this process")
def test_linear_on_two_devices_in_one_process():
    from comfyui_turing_utils_kernel import _C, _lib

    g = torch.Generator().manual_seed(81)
    m, k, n = 300, 5120, 264
    x = (torch.randn((m, k), generator=g)).to(torch.bfloat16)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    xb = x.view(torch.int16).numpy().view(np.uint16)
    ref = oracle.convrot_w8a8_linear(xb, w.numpy(), w_s.numpy(), bias.numpy())
    for dev in (torch.device("cuda", 0), torch.device("cuda", 1)):
        with torch.cuda.device(dev):
            q, s = _C.turing_bf16_int8_convrot_quantize(x.to(dev), 256, False)
            out = _C.turing_int8_linear(q, w.to(dev), s, w_s.to(dev), bias.to(dev))
            torch.cuda.synchronize(dev)
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref), dev
        assert _lib.device_error(dev.index, clear=True) == 0
