"""Generate the golden fixtures in ``tests/golden/*.npz`` from the reference implementation.

Run in a container where the reference checkout is importable (it is not needed afterwards;
the GPU box never runs this):

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

For each case in ``cases.CASES`` it runs the reference's ``tattn.reference.tiled_forward``
(src/tattn/reference.py:29-64), ``tiled_backward`` (reference.py:67-102) and, for config 1,
``naive_attention`` (reference.py:18-26) with torch autograd, on CPU, and stores:

  o, m, dq, dk, dv                      -- the tiled reference's outputs
  o_naive, dq_naive, dk_naive, dv_naive -- config 1 only: the fp32 definition + autograd
  meta                                  -- JSON: case parameters and input digests
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.cases import CASES, digest, make_inputs  # noqa: E402


def main() -> None:
    from tattn.reference import naive_attention, tiled_backward, tiled_forward  # the reference

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, case in CASES.items():
        q, k, v, do = make_inputs(case)
        o, m = tiled_forward(q, k, v, case.causal, case.sm_scale)
        dq, dk, dv = tiled_backward(q, k, v, o, m, do, case.causal, case.sm_scale)
        out = {
            "o": o.numpy(), "m": m.numpy(),
            "dq": dq.contiguous().numpy(), "dk": dk.contiguous().numpy(), "dv": dv.contiguous().numpy(),
        }  # fmt: skip
        if name.startswith("cfg1"):
            qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
            ref = naive_attention(qr, kr, vr, causal=case.causal, sm_scale=case.sm_scale)
            ref.backward(do.float())
            out.update(
                o_naive=ref.detach().numpy(), dq_naive=qr.grad.numpy(),
                dk_naive=kr.grad.numpy(), dv_naive=vr.grad.numpy(),
            )  # fmt: skip
        meta = {
            "shape": list(case.shape), "dtype": case.dtype, "causal": case.causal,
            "seeds": list(case.seeds), "layout": case.layout, "sm_scale": case.sm_scale,
            "digests": [digest(t) for t in (q, k, v, do)],
            "generator": "tattn.reference (src/tattn/reference.py) on CPU, torch " + torch.__version__,
        }  # fmt: skip
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array(json.dumps(meta)),
            **{kk: np.ascontiguousarray(vv) for kk, vv in out.items()},
        )
        print(name, {kk: vv.shape for kk, vv in out.items()})


if __name__ == "__main__":
    main()
