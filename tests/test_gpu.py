"""GPU tests (B200): kernels against fp32/fp64 PyTorch references and the
CUDA paths of the backend through torch.distributed."""

import os
import subprocess
import sys

import pytest
import torch

from mp import check, run

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = {"CMX_DEVICE": "cuda"}


def ngpu():
    return torch.cuda.device_count()


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("shape", [(20, 20, 20), (37, 45, 71), (132, 68, 36)])
def test_jacobi7_matches_reference(dtype, shape):
    from commux_b200.ops import jacobi7, jacobi7_reference

    h = 2
    g = torch.Generator().manual_seed(3)
    u = torch.rand(shape, generator=g, dtype=torch.float64) * 2 - 1
    v_ref = torch.zeros_like(u)
    r_ref = jacobi7_reference(u, v_ref, h)
    ud = u.to(dtype).cuda()
    vd = torch.zeros_like(ud)
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    jacobi7(ud, vd, h, res)
    torch.cuda.synchronize()
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    got = vd.double().cpu()[h:-h, h:-h, h:-h]
    assert torch.allclose(got, v_ref[h:-h, h:-h, h:-h], rtol=tol, atol=tol)
    assert abs(float(res) - r_ref) <= (1e-9 if dtype == torch.float64 else 1e-3) * max(1.0, r_ref)
    # the ghost shell of v is untouched
    assert float(vd[:h].abs().sum()) == 0.0


def test_p2p_self_sends():
    check(run("gpu_p2p.py", 1, env=CUDA))


def test_p2p_self_sends_group_window():
    check(run("gpu_p2p.py", 1, env=dict(CUDA, COMMUX_GROUP="1")))


def test_p2p_two_ranks():
    # one GPU: both ranks share it (host-gated path); more: one GPU per rank
    check(run("gpu_p2p.py", 2, env=CUDA, timeout=180))


def test_torch_dist_cuda():
    check(run("torch_dist.py", 2, env=CUDA, timeout=180))


def test_coalesce_cuda():
    check(run("coalesce.py", 2, env=dict(CUDA, COMMUX_COALESCE="1", COMMUX_GROUP="1"), timeout=180))


@pytest.mark.parametrize("world", [1, 2])
def test_halo_cuda(world):
    check(run("halo.py", world, env=dict(CUDA, COMMUX_GROUP="1"), timeout=180))


def test_collectives_cuda():
    check(run("collectives.py", 2, env=dict(CUDA, CMX_A2A="1"), timeout=240))


@pytest.mark.parametrize("variant", ["default", "nvls", "p2p", "twoshot"])
def test_collective_numerics_cuda(variant):
    # every rank on its own GPU where there are enough (NVLS and peer kernels),
    # else ranks share GPUs (host-staged path); "nvls" forces the multicast
    # path at any rank count and size, "p2p" turns it off
    world = max(2, min(ngpu(), 8))
    env = dict(CUDA)
    if variant == "nvls":
        env.update(COMMUX_NVLS_MIN_RANKS="2", COMMUX_NVLS_MIN_BYTES="0")
    elif variant == "p2p":
        env.update(COMMUX_NVLS="0")
    elif variant == "twoshot":
        env.update(COMMUX_NVLS="0", COMMUX_ALGO="twoshot")
    check(run("gpu_coll_numerics.py", world, env=env, timeout=600))


def test_smoke_entry():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "__graft_entry__.py")], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


def test_plan_self():
    check(run("gpu_plan.py", 1, env=CUDA))


def test_plan_two_ranks():
    # shared GPU: host-gated per start; one GPU per rank: device flags
    check(run("gpu_plan.py", 2, env=CUDA, timeout=180))


@pytest.mark.parametrize("world", [1, 2])
def test_halo_cuda_batch_path(world):
    check(run("halo.py", world, env=dict(CUDA, COMMUX_HALO_PLAN="0", COMMUX_GROUP="1"), timeout=180))


def test_ipc_mappings_bounded_under_allocator_churn():
    # ranks share one GPU or have one each: either way the receiver maps the
    # sender's segments through CUDA IPC
    check(run("gpu_ipc_churn.py", 2, env=CUDA, timeout=240))


def test_unexportable_memory_staged():
    # the caching allocator's expandable segments cannot be exported through
    # CUDA IPC: sends to another process travel through the export pool
    env = dict(CUDA, PYTORCH_CUDA_ALLOC_CONF="expandable_segments:True")
    check(run("gpu_p2p.py", 2, env=dict(env, CMX_EXPECT_EXPORT_STAGING="1"), timeout=240))
    check(run("gpu_plan.py", 2, env=env, timeout=240))
    check(run("halo.py", 2, env=dict(env, COMMUX_GROUP="1"), timeout=240))


def test_tcp_cuda_p2p_staged():
    # ranks "on other hosts" (forced TCP): CUDA tensors travel through host memory
    check(run("gpu_p2p.py", 2, env=dict(CUDA, COMMUX_TRANSPORT="tcp"), timeout=240))


def test_tcp_cuda_collectives_staged():
    check(run("collectives.py", 2, env=dict(CUDA, COMMUX_TRANSPORT="tcp", CMX_A2A="1"), timeout=240))


def test_device_bounds_checks():
    """The bounds-check build (kernels test every unit against the limits the
    host derived, and report instead of touching memory outside them) passes
    its self-test; the production library has the checks compiled out."""
    lib = os.path.join(ROOT, "build-devchecks", "lib", "libcommux_cuda.so")
    if not os.path.exists(lib):
        r = subprocess.run([sys.executable, "-m", "commux_b200.build", "--device-checks"], cwd=ROOT,
                           capture_output=True, text=True, timeout=1200)
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    worker = os.path.join(ROOT, "tests", "workers", "device_checks.py")
    prod = os.path.join(ROOT, "commux_b200", "lib", "libcommux_cuda.so")
    for which, path in (("checked", lib), ("production", prod)):
        r = subprocess.run([sys.executable, worker, which, path], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
