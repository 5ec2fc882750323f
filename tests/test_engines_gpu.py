"""Every QMM engine the library ships, forced on one at a time, against the oracle.

The planner picks the streaming engine (qmm_st.cu, mma.sync consumers) for every shape with
K % 512 == 0; the other engines are selected by environment switches read when a plan is made:
DSPARK_QMM_ST_TC=1 (streaming engine with tcgen05 consumers: weights dequantized into tensor
memory, MMA with A in TMEM), DSPARK_QMM_IMPL=tc (the tcgen05 engine of qmm_tc.cu) and
DSPARK_QMM_IMPL=mma (per-tile CTAs, qmm.cu; also the path of K % 512 != 0). Plans are cached per
process, so each engine runs in a fresh interpreter. Each checks 1/16/32 rows, 4- and 8-bit,
one plain and one deep-K shape, against the oracle (max |diff| <= 1e-2 * max|ref|) and that the
device status stays clean.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

_SCRIPT = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, {root!r})
sys.path.insert(0, {oracle!r})
import oracle
import mlx_dspark_b200
from mlx_dspark_b200 import _lib, skinny_qmm
dev = torch.device("cuda", 0)
_lib.ensure_init(0)
rng = np.random.default_rng(7)
worst = 0.0
for (N, K) in ((1024, 4096), (512, 12288), (776, 1536)):
    for bits in (4, 8):
        wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), bits)
        W = [torch.from_numpy(wq.view(np.int32)).to(dev),
             torch.from_numpy(sc.view(np.int16)).view(torch.bfloat16).to(dev),
             torch.from_numpy(bi.view(np.int16)).view(torch.bfloat16).to(dev)]
        for M in (1, 16, 32):
            x = oracle.to_bf16(rng.normal(0, 1, (M, K)))
            y = skinny_qmm.qmm(torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev),
                               *W, bits)
            ref = oracle.qmm(x, wq, sc, bi, bits)
            err = float(np.abs(y.float().cpu().numpy() - ref).max())
            tol = 1e-2 * max(float(np.abs(ref).max()), 1.0)
            assert err <= tol, (N, K, bits, M, err, tol)
            worst = max(worst, err / tol)
st = _lib.device_status(0)
assert st == 0, hex(st)
print("engine ok, worst err/tol", round(worst, 4))
"""


@pytest.mark.parametrize("env", [{"DSPARK_QMM_ST_TC": "1"}, {"DSPARK_QMM_IMPL": "tc"},
                                 {"DSPARK_QMM_IMPL": "mma"}],
                         ids=["st-tcgen05", "tc", "mma"])
def test_forced_engine_matches_oracle(env):
    e = dict(os.environ, **env)
    code = _SCRIPT.format(root=str(ROOT), oracle=str(ROOT / "oracle"))
    r = subprocess.run([sys.executable, "-c", code], env=e, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "engine ok" in r.stdout
