"""Stream order of the device entry point.

The top-k sampling kernel is launched as a programmatic dependent of whatever
precedes it on the stream: its launch may overlap the producer's end, and it
must read nothing before the producer's writes are visible. Here a kernel
writes the logits (and the uniforms) on the stream immediately before the call,
with no synchronisation in between, and the tokens must equal the oracle's.
"""
import numpy as np
import pytest

from neuraval_b200 import native, workloads
from tests.gpu_util import assert_exact, run_oracle

pytestmark = pytest.mark.gpu


def test_inputs_written_by_the_previous_kernel(gpu_sampler, oracle):
    import torch
    wl = workloads.zipf_ranked(B=64, V=50000, H=256, seed=41)
    B, V = wl["logits"].shape
    base = torch.from_numpy(wl["logits"]).cuda()
    hist = torch.from_numpy(wl["hist_ids"]).cuda()
    offs = torch.from_numpy(wl["hist_offsets"]).cuda()
    ubase = torch.from_numpy(wl["uniforms"]).cuda()
    params = native.make_params(**wl["params"])
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    torch.cuda.synchronize()
    for trial in range(4):
        # fresh buffers holding stale values: reading them early gives other tokens
        logits = torch.full_like(base, 7.0)
        u = torch.full_like(ubase, 0.5)
        tokens = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        flags = torch.zeros(B, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        # elementwise kernels produce the inputs; the call follows on the same stream
        torch.add(base, 0.0, out=logits)
        torch.add(ubase, 0.0, out=u)
        gpu_sampler.sample_rows_device(logits, hist, offs, u, params, tokens, flags)
        torch.cuda.synchronize()
        assert_exact(tokens.cpu().numpy(), flags.cpu().numpy().astype(np.uint32), ot, of,
                     f"stream order, trial {trial}")
