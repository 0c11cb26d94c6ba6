"""The reference model's own calls, replayed through this library's fused-ops module (GPU).

``tests/golden/binding_trace.npz`` (``make_golden.py``, ``QW_GOLDEN_ONLY=binding``) holds
every call that the reference's ``FusedTargetModel`` makes through the reference's
``ModuleFusedOps`` on the tiny configuration -- a 16-token prefill and one decode step
(model/qwen35_moe_dflash/fused/model.py:217-300, bound by fused/ops.py:138-176) --
recorded at the adapter-module boundary: the operator, its arguments exactly as the
model passes them (positional and keyword, dtypes and shapes, weights by name) and the
reference backend's outputs.  Each call is replayed here through
``qwen35_dflash_b200.fused_ops`` on the GPU with the recorded inputs, and its outputs are
compared with the recorded ones within the tolerances of the operator golden tests
(fp16: rounding to the output dtype, a few ulps where the summation order differs).
The module also meets the checks ``ModuleFusedOps`` makes when it binds an adapter.
"""
import json
import types

import numpy as np
import pytest
import torch

from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

U16 = 2 ** -11   # fp16 ulp at 1

# (atol, rtol) per operator; None: bit-exact (copies and concatenations)
TOL = {
    "rms_norm": (1e-6, 2 * U16),
    "conv_state_update": None,
    "causal_conv1d": (1e-6, 2 * U16),
    "chunk_gated_delta_rule": (2e-3, 2e-2),
    "cache_update": None,
    "attention": (4 * U16, 4 * U16),
    "moe": (4 * U16, 4 * U16),
}


def _tiny_weights():
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from oracle.numerics import quantize_w4, dequantize_w4
    cfg = qcfg.TINY
    out = {}
    for name, value in synthetic.init_weights(cfg, seed=17).items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        out[name] = torch.from_numpy(value).to(torch.float16).cuda()
    return out


def test_module_meets_the_binding_checks(cuda_lib):
    from qwen35_dflash_b200 import fused_ops as Q
    assert isinstance(Q, types.ModuleType)
    assert type(Q.FUSED_OPS_ABI) is int and Q.FUSED_OPS_ABI == 1
    assert isinstance(Q.BACKEND_ID, str) and Q.BACKEND_ID.strip()
    assert Q.IS_REFERENCE_BACKEND is False
    for name in TOL:
        assert callable(getattr(Q, name, None)), name


def test_reference_model_calls_replay(golden, cuda_lib):
    from qwen35_dflash_b200 import fused_ops as Q
    d = golden("binding_trace.npz")
    calls = json.loads(str(d["calls"]))
    assert len(calls) > 0 and {c["op"] for c in calls} == set(TOL)
    weights = _tiny_weights()

    def dec(e):
        if "weight" in e:
            return weights[e["weight"]]
        if "array" in e:
            return torch.from_numpy(np.ascontiguousarray(d[e["array"]])).cuda().to(getattr(torch, e["dtype"]))
        if "seq" in e:
            return tuple(dec(x) for x in e["seq"])
        return e["value"]

    def outputs(e):
        if "seq" in e:
            return [x for s in e["seq"] for x in outputs(s)]
        return [e]

    for i, c in enumerate(calls):
        args = [dec(a) for a in c["args"]]
        kwargs = {k: dec(v) for k, v in c["kwargs"].items()}
        got = getattr(Q, c["op"])(*args, **kwargs)
        got = list(got) if isinstance(got, tuple) else [got]
        want = outputs(c["out"])
        assert len(got) == len(want), (i, c["op"])
        for j, (g, w) in enumerate(zip(got, want)):
            what = f"call {i} {c['op']} output {j}"
            assert str(g.dtype).replace("torch.", "") == w["dtype"], what
            ref = d[w["array"]]
            assert tuple(g.shape) == ref.shape, (what, tuple(g.shape), ref.shape)
            if TOL[c["op"]] is None:
                np.testing.assert_array_equal(to_np(g), ref, err_msg=what)
            else:
                assert_close(to_np(g), ref, *TOL[c["op"]], what=what)
