"""The reference's own GPU schedule (its CUDA kernels and cuBLAS FP32 op
sequence, oracle/ref_gpu.py) runs on the B200 and agrees with the C oracle of
its CPU backend -- which checks the restated schedule -- and is timed beside
this engine on the 16384-token forward.  Needs oracle/_ref/libref_gpu.so,
built here from the reference tree (oracle/ref_gpu_build.py)."""
import json
import os

import numpy as np
import pytest

from laya_rust_b200 import engine as E
from laya_rust_b200 import modelgen, workloads

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def setup():
    from oracle import ref_gpu
    from oracle.oracle import OracleModel
    if not ref_gpu.available():
        pytest.skip("oracle/_ref/libref_gpu.so was not built (no reference tree where the library was built)")
    path = modelgen.cached_model(seed=0)
    om = OracleModel(path)
    rg = ref_gpu.RefGpuSchedule(om)
    yield om, rg
    rg.close()
    om.close()


def test_reference_schedule_matches_the_cpu_oracle(setup):
    om, rg = setup
    fx = json.load(open(os.path.join(HERE, "golden", "fixture_requests.json")))
    for f in fx:
        for fw in f["forwards"]:
            args = (fw["n"], fw["l"], fw["k"], fw["ids"], fw["att"], fw["mpos"], fw["mmask"], fw["qtype"])
            gl, ga = rg.forward(*args)
            wl, wa = om.forward(*args)
            assert np.abs(gl - wl).max() <= 2e-3 + 1e-3 * np.abs(wl).max(), f["name"]
            assert np.abs(ga - wa).max() <= 2e-3 + 1e-3 * np.abs(wa).max(), f["name"]


def test_reference_schedule_timed_beside_the_engine(setup):
    om, rg = setup
    req = workloads.forward_16k(0)
    ref_ms = rg.time(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype, 3)
    eng = E.Engine(modelgen.cached_model(seed=0), device=0)
    p = eng.plan(req)
    p.capture()
    import torch
    s = torch.cuda.ExternalStream(eng.stream())
    for _ in range(3):
        p.run()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s)
    for _ in range(10):
        p.run()
    t1.record(s)
    torch.cuda.synchronize()
    ours = t0.elapsed_time(t1) / 10
    real = workloads.real_tokens(req)
    print(f"reference GPU schedule: {ref_ms:.1f} ms per forward ({real / ref_ms * 1e3:.0f} real tok/s); "
          f"this engine: {ours:.2f} ms ({real / ours * 1e3:.0f} real tok/s); {ref_ms / ours:.1f}x")
    p.close()
    eng.close()
    assert ours < ref_ms
