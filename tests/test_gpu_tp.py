"""Tensor-parallel MLP on 2 GPUs (skipped with fewer): every exchange against
the single-GPU block, and the copy-engine exchange's bounded wait when a rank
leaves between steps. Each case runs tests/tp_worker.py under torchrun with
NVLS off (NCCL_NVLS_ENABLE=0); the exchange itself maps peer memory with plain
CUDA IPC handles, so no multicast object is ever bound."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _run(mode, port, nproc=2):
    if _gpus() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_DEVICE_MAX_CONNECTIONS="32")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(nproc),
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "tp_worker.py"), mode]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")]
    assert r.returncode == 0 and lines, r.stdout[-3000:] + r.stderr[-3000:]
    return json.loads(lines[-1][len("RESULT "):])


@pytest.mark.parametrize("nproc", [2, 4])
def test_tp_exchanges_match_single_gpu(nproc):
    res = _run("parity", 29711 + nproc, nproc)
    print(res)
    for name in ("copy_engine", "copy_engine_gemm1_chunked", "copy_engine_one_stream", "nccl",
                 "peer_store"):
        # the only change from one GPU is the fp32 summation order of the partials
        assert res[name]["bit_exact"] >= 0.93, (name, res[name])
        assert res[name]["max_err_over_scale"] <= 2.0 ** -6, (name, res[name])
        # each rank's row block arrives (own reduce and every peer's pulled rows)
        assert min(res[name + "_blocks_exact"]) >= 0.9, (name, res[name + "_blocks_exact"])
    assert res["copy_engine_joined_streams"] == 2 * (nproc - 1) + 2
    assert res["copy_engine_one_stream_joined_streams"] == 4
    assert res["ranks_agree"]
    assert res["ce_eq_one_stream"] and res["ce_eq_peer_store"] and res["ce_eq_gemm1_chunked"]
    assert res["device_error"] == 0


def test_tp_copy_engine_timeout_when_a_rank_leaves():
    res = _run("timeout", 29713)
    print(res)
    assert res["raised"], res
    assert res["context_ok"] and res["device_error"] == 0
