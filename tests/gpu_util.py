"""Helpers shared by the GPU parity tests (inputs as CUDA tensors, tolerances)."""
import numpy as np
import torch

# rel-L2 bounds against the float64 oracle on the same (dtype-rounded) inputs.
TOL = {"f32": 1e-4, "bf16": 1e-2}

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16}


def to_dev(a, dtype="f32", int32=False):
    if a is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(a))
    if int32:
        return t.to(torch.int32).cuda()
    return t.to(TORCH_DT[dtype]).cuda()


def dev_inputs(inp, dtype):
    """x, dt, B, C, z in the input dtype; A, D, dt_bias, init f32; seq_idx/cu int32."""
    d = {}
    for k in ("x", "dt", "B", "C", "z"):
        d[k] = to_dev(inp[k], dtype)
    for k in ("A", "D", "dt_bias", "initial_states"):
        d[k] = to_dev(inp[k], "f32")
    d["seq_idx"] = to_dev(inp["seq_idx"], int32=True)
    d["cu_seqlens"] = to_dev(inp["cu_seqlens"], int32=True)
    return d


def rel_l2(got, ref):
    g = got.detach().double().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    den = np.linalg.norm(r.ravel())
    return float(np.linalg.norm((g - r).ravel()) / (den if den > 0 else 1.0))
