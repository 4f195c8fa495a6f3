"""Output tolerances of the GPU parity tests.

* fp32 outputs: elementwise ``|out - ref| <= 1e-5 + 1e-5 |ref|``.
* bf16 / fp16 outputs: the stated bound is 2e-3 relative, measured in the L2
  norm over the output tensor: ``||out - ref|| / ||ref|| <= 2e-3``.  In
  addition every element must be within one rounding to the output type of
  the exact value: ``|out - ref| <= u |ref| (1 + 1e-2) + 1e-5`` with unit
  roundoff ``u = 2^-8`` (bf16) or ``2^-11`` (fp16).  An elementwise
  2e-3 bound cannot hold for bf16 outputs: rounding alone reaches 2^-8 = 3.9e-3.

``ref`` is the float64 oracle evaluated on the same (already rounded) inputs.
"""

import numpy as np
import torch

UNIT_ROUNDOFF = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def assert_output_close(out, ref, dtype=None):
    dtype = dtype or out.dtype
    o = out.double().cpu().numpy() if isinstance(out, torch.Tensor) else np.asarray(out, np.float64)
    r = ref.double().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, np.float64)
    err = np.abs(o - r)
    if dtype == torch.float32:
        bad = err > 1e-5 + 1e-5 * np.abs(r)
        assert not bad.any(), f"fp32: {bad.sum()} elements off, max err {err.max():.3e}"
        return
    u = UNIT_ROUNDOFF[dtype]
    rel = np.linalg.norm(o - r) / max(np.linalg.norm(r), 1e-300)
    assert rel <= 2e-3, f"{dtype}: relative L2 error {rel:.3e} > 2e-3"
    bad = err > u * np.abs(r) * 1.01 + 1e-5
    assert not bad.any(), f"{dtype}: {bad.sum()} elements beyond one rounding, max err {err.max():.3e}"
