"""The reference's own JointTransformerBlock (src_ii/transformer.py:588-717) run
unmodified on this library through the sys.modules swap of INTEGRATION.md,
against the same block on the reference's Triton kernels.

Needs the reference package next to the repository (``baseline/_ref``: its
``futudiffu/`` and ``src_ii/`` directories, as a pip install would lay them
out); skipped where it is absent.  ``tests/golden/dropin_block.py`` does the
work, each side in a fresh interpreter.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not (REF / "src_ii" / "transformer.py").exists(), reason="reference package not in baseline/_ref")
def test_reference_block_on_swapped_modules(cuda_device):
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import dropin_block

    rec = dropin_block.compare(REF)
    assert rec["kernels"] == {"reference": "futudiffu.fp8_kernels", "swapped": "futudiffu_b200.fp8_kernels"}
    assert rec["finite"]
    # the DiT block gate: INT8 / FP8 code flips of the two kernel sets move single
    # outputs by a few bf16 ulps
    assert rec["cosine"] >= 0.9999, rec
    assert rec["max_abs_err"] <= 0.05 * rec["max_abs_ref"] + 0.01, rec
