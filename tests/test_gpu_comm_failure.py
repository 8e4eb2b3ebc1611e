"""GPU, one device: failure detection of the gradient exchange, made on the
host (no GPU fault).  A communicator of two ranks whose second rank never
joins must not hold the process: ne_comm_init gives up at the exchange's
deadline (ne_comm_set_timeout) with NE_ERR_TIMEOUT, after aborting the
non-blocking NCCL initialisation, and the context stays usable for GPU work.
The rank that never joins is simply never started.  The call runs in a child
process with NVLS off, bounded by a process timeout as the last resort."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys, time
sys.path.insert(0, sys.argv[1])
import numpy as np
import torch
import neural_engine_b200 as ne
e = ne.Engine(ne.ModelConfig(1, 128, 256, 2, 2, 64, 256), device=0)
e.comm_set_timeout(3000)
uid = ne.Engine.comm_unique_id()
t0 = time.time()
res = {"status": 0}
try:
    e.comm_init(uid, 0, 2)            # rank 1 of 2 never starts
except ne.NeError as err:
    res["status"] = err.status
    res["msg"] = str(err)
res["seconds"] = time.time() - t0
# the context still runs kernels: a small product against float64
a = (torch.randn(128, 128) * 0.1).to(torch.bfloat16)
b = (torch.randn(64, 128) * 0.1).to(torch.bfloat16)
da, db = a.cuda(), b.cuda()
out = torch.zeros(128, 64, device="cuda")
e.gemm_device(da.data_ptr(), 128, 128, db.data_ptr(), 128, 64, 128, 1, out.data_ptr(), 64)
e.sync()
res["gemm_err"] = float((out.cpu().double() - a.double() @ b.double().T).abs().max())
e.close()
print("RESULT " + json.dumps(res), flush=True)
"""


def test_comm_init_times_out_when_a_rank_never_joins():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NCCL_DEBUG="WARN")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True,
                       timeout=180, env=env, cwd=ROOT)
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")]
    assert r.returncode == 0 and line, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(line[0][7:])
    assert res["status"] == 6, res          # NE_ERR_TIMEOUT
    assert 2.5 <= res["seconds"] <= 60, res
    assert "every rank must join" in res["msg"], res
    assert res["gemm_err"] <= 1e-3, res
