"""Failure detection of the tensor-parallel group, made on the host: a rank whose peers never
join.  One process asks to be rank 0 of a 2-rank group and nobody else comes; every wait on
the peers is bounded (IAM_TP_TIMEOUT_S), so creating the model must end with IAM_ERR_TIMEOUT
within seconds instead of blocking forever.  Nothing on the GPU faults or hangs: the only
waits are host-side polls of the NCCL communicator.  Runs in a child process so that the
environment variable and the aborted communicator stay out of the test session.
"""
import os
import subprocess
import sys
import time

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys, time
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
from conftest import load_pkg
iam = load_pkg()
cfg = iam.ModelConfig.make(dim=256, n_layers=1, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512,
                           max_ctx=64)
t0 = time.time()
try:
    iam.Model.random(cfg, seed=1, device=0, tp=(0, 2, iam.tp_unique_id()))
    print("UNEXPECTED: created")
except iam.IamError as e:
    print("CODE", e.code, "AFTER", round(time.time() - t0, 1))
"""


@pytest.mark.timeout(120)
def test_missing_peer_ends_in_timeout(iam, cuda):
    env = dict(os.environ, IAM_TP_TIMEOUT_S="3")
    src = CHILD.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    t0 = time.time()
    r = subprocess.run([sys.executable, "-c", src], env=env, capture_output=True, text=True, timeout=100)
    took = time.time() - t0
    line = [ln for ln in r.stdout.splitlines() if ln.startswith(("CODE", "UNEXPECTED"))]
    assert line, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    assert line[-1].startswith("CODE"), line
    code = int(line[-1].split()[1])
    assert code == iam.IAM_ERR_TIMEOUT, (line, r.stderr[-1000:])
    assert took < 90, took


def test_exchange_wait_runs_out_on_one_gpu(iam, cuda):
    """The bounded device-side wait of the one-shot exchanges, driven to its limit on one GPU:
    a two-rank exchange window whose second rank is a local buffer that never sends.  The
    first all-reduce gives up after spin_limit polls per element and sets the error word; the
    next one returns without waiting; the status is IAM_ERR_TIMEOUT, as iam_model_status
    reports it for a model.  No fault and no hang: every wait has its poll bound."""
    rc, err, first_ms, second_ms = iam.tp_wait_selftest(n=256, spin_limit=4096)
    assert rc == iam.IAM_ERR_TIMEOUT, (rc, err)
    assert err == 1
    assert 0.0 < first_ms < 2000.0, first_ms
    assert second_ms < first_ms, (first_ms, second_ms)
    # a longer bound waits longer before it gives up
    rc2, err2, first2, _ = iam.tp_wait_selftest(n=256, spin_limit=4 * 4096)
    assert rc2 == iam.IAM_ERR_TIMEOUT and err2 == 1
    assert first2 > first_ms, (first_ms, first2)
