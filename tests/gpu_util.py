"""Helpers shared by the GPU parity tests (run the kernels, run the oracle, compare)."""
from __future__ import annotations

import numpy as np

from neuraval_b200 import native

# EXP_SLOW records which path computed a weight; the oracle also evaluates
# weights the kernels provably never need, so that bit is not compared.
COMPARED_FLAGS = ~native.FLAG_EXP_SLOW & 0xFFFFFFFF


def to_dev(wl, offset=0):
    """Device copies of a workload; `offset` floats of padding before the logits
    make the row base pointer deliberately unaligned."""
    import torch
    lg = wl["logits"]
    if offset:
        flat = torch.zeros(lg.size + offset, dtype=torch.float32, device="cuda")
        flat[offset:] = torch.from_numpy(lg.reshape(-1)).cuda()
        logits = flat[offset:].view(lg.shape)
    else:
        logits = torch.from_numpy(lg).cuda()
    hist = torch.from_numpy(np.ascontiguousarray(wl["hist_ids"], dtype=np.int32)).cuda()
    if hist.numel() == 0:
        hist = torch.zeros(1, dtype=torch.int32, device="cuda")
    offs = torch.from_numpy(np.ascontiguousarray(wl["hist_offsets"], dtype=np.int32)).cuda()
    u = torch.from_numpy(np.ascontiguousarray(wl["uniforms"], dtype=np.float32)).cuda()
    return logits, hist, offs, u


def run_gpu(sampler, wl, want_probs=False, offset=0, params=None):
    import torch
    logits, hist, offs, u = to_dev(wl, offset)
    B, V = wl["logits"].shape
    tokens = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    flags = torch.zeros(B, dtype=torch.int32, device="cuda")
    probs = torch.full((B, V), -1.0, dtype=torch.float32, device="cuda") if want_probs else None
    p = params if params is not None else native.make_params(**wl["params"])
    sampler.sample_rows_device(logits, hist, offs, u, p, tokens, flags, probs)
    torch.cuda.synchronize()
    return (tokens.cpu().numpy(), flags.cpu().numpy().astype(np.uint32),
            probs.cpu().numpy() if want_probs else None)


def run_oracle(oracle, wl, exp_mode, want_probs=False, threads=16):
    p = oracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], dtype=np.int64)
    return oracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], p,
                              exp_mode=exp_mode, threads=threads, want_probs=want_probs)


def assert_exact(gt, gf, ot, of, label=""):
    """Bit-exact agreement with the oracle in correctly-rounded-exp mode."""
    bad = np.nonzero((gt != ot) | ((gf & COMPARED_FLAGS) != (of & COMPARED_FLAGS)))[0]
    assert bad.size == 0, (f"{label}: {bad.size} rows differ, first {bad[:8]} "
                           f"gpu {gt[bad[:8]]}/{gf[bad[:8]]} oracle {ot[bad[:8]]}/{of[bad[:8]]}")


def parity_report(gt, gf, ot, of):
    """Token parity against the reference arithmetic (libm expf): rows may differ
    only where a boundary/tie flag is set (on either side)."""
    exempt = ((gf | of) & native.PARITY_EXEMPT) != 0
    differ = gt != ot
    return dict(rows=int(gt.size), flagged=int(exempt.sum()),
                differ_unflagged=int((differ & ~exempt).sum()),
                differ_flagged=int((differ & exempt).sum()))
