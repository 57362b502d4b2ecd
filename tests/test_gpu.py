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


# Counter conditions (CMX_EXPECT, checked by every worker at exit) that
# prove which path ran. "peer": every rank on its own GPU, so p2p completes
# through device flags (the sender waits on its stream, the receiver pulls
# over NVLink) and collectives run the device kernels. "shared": every rank
# on GPU 0, so p2p completes through host FINs and collectives are staged
# through the host (kernels of two processes on one GPU never wait on each
# other).
# (A first send to a peer whose GPU is not yet known may still complete by a
# host FIN, so the peer form does not require zero of those.)
PEER_P2P = "cuda_sends_device_flag>0,cuda_pulls_peer_gpu>0,cuda_pulls_same_gpu==0"
SHARED_P2P = "cuda_sends_host_fin>0,cuda_pulls_same_gpu>0,cuda_sends_device_flag==0,cuda_pulls_peer_gpu==0"
PEER_PLAN = "cuda_plan_device_msgs>0,cuda_plan_shared_msgs==0,cuda_plan_starts>0"
SHARED_PLAN = "cuda_plan_shared_msgs>0,cuda_plan_device_msgs==0,cuda_plan_starts>0"
PEER_COLL = "coll_shared_gpu==0,coll_calls>0"
SHARED_COLL = "coll_shared_gpu==1"


def topology(mode, world, expect):
    """Environment of a multi-rank CUDA test in one topology; skips the peer
    form where the box has fewer GPUs than ranks (it would silently run the
    shared form instead)."""
    if mode == "peer":
        if ngpu() < world:
            pytest.skip(f"peer-GPU path needs {world} GPUs, one per rank; this box has {ngpu()}")
        return dict(CUDA, CMX_EXPECT=expect[0])
    return dict(CUDA, CMX_SHARED_GPU="1", CMX_EXPECT=expect[1])


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("shape", [(20, 20, 20), (37, 45, 71), (132, 68, 36), (7, 9, 11)])
def test_jacobi7_core_plus_shell_is_whole(dtype, shape):
    # the overlapped step's two updates write exactly the whole-interior update
    from commux_b200.ops import jacobi7, jacobi7_reference

    h = 2
    g = torch.Generator().manual_seed(5)
    u = (torch.rand(shape, generator=g, dtype=torch.float64) * 2 - 1).to(dtype).cuda()
    whole, parts = torch.zeros_like(u), torch.zeros_like(u)
    r_whole = torch.zeros(1, dtype=torch.float64, device="cuda")
    r_parts = torch.zeros(1, dtype=torch.float64, device="cuda")
    jacobi7(u, whole, h, r_whole)
    jacobi7(u, parts, h, r_parts, part="core")
    core_only = parts.clone()
    jacobi7(u, parts, h, r_parts, part="shell")
    torch.cuda.synchronize()
    assert torch.equal(whole, parts)
    # the core part leaves the one-cell boundary layer alone
    assert float(core_only[h, h:-h, h:-h].abs().sum()) == 0.0
    assert float(core_only[h:-h, h:-h, -h - 1].abs().sum()) == 0.0
    v_ref = torch.zeros(shape, dtype=torch.float64)
    r_ref = jacobi7_reference(u.double().cpu(), v_ref, h)
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    assert torch.allclose(parts.double().cpu()[h:-h, h:-h, h:-h], v_ref[h:-h, h:-h, h:-h], rtol=tol, atol=tol)
    assert abs(float(r_parts) - float(r_whole)) <= 1e-9 * max(1.0, abs(r_ref))


def test_overlapped_steps_match_sequential():
    check(run("halo_overlap.py", 1, env=CUDA, timeout=240))


def test_p2p_self_sends():
    check(run("gpu_p2p.py", 1, env=CUDA))


def test_p2p_self_sends_group_window():
    check(run("gpu_p2p.py", 1, env=dict(CUDA, COMMUX_GROUP="1")))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_p2p_two_ranks(mode):
    check(run("gpu_p2p.py", 2, env=topology(mode, 2, (PEER_P2P, SHARED_P2P)), timeout=180))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_torch_dist_cuda(mode):
    env = topology(mode, 2, (PEER_P2P + "," + PEER_COLL, SHARED_P2P + "," + SHARED_COLL))
    check(run("torch_dist.py", 2, env=env, timeout=180))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_coalesce_cuda(mode):
    env = topology(mode, 2, (PEER_P2P, SHARED_P2P))
    check(run("coalesce.py", 2, env=dict(env, COMMUX_COALESCE="1", COMMUX_GROUP="1"), timeout=180))


def test_halo_cuda_one_rank():
    check(run("halo.py", 1, env=dict(CUDA, COMMUX_GROUP="1", CMX_EXPECT="cuda_plan_starts>0"), timeout=180))


@pytest.mark.parametrize("mode,world", [("peer", 2), ("peer", 4), ("peer", 8), ("shared", 2)])
def test_halo_cuda(mode, world):
    env = topology(mode, world, (PEER_PLAN, SHARED_PLAN))
    check(run("halo.py", world, env=dict(env, COMMUX_GROUP="1"), timeout=300))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_collectives_cuda(mode):
    env = topology(mode, 2, (PEER_COLL, SHARED_COLL))
    check(run("collectives.py", 2, env=dict(env, CMX_A2A="1"), timeout=240))


COLL_VARIANTS = {
    # env, counters that prove the variant's kernels ran
    "default": ({}, "coll_oneshot>0,coll_twoshot>0"),
    "nvls": ({"COMMUX_NVLS_MIN_RANKS": "2", "COMMUX_NVLS_MIN_BYTES": "0"}, "coll_nvls_enabled==1,coll_nvls>0"),
    "p2p": ({"COMMUX_NVLS": "0"}, "coll_nvls_enabled==0,coll_nvls==0,coll_oneshot>0,coll_twoshot>0"),
    "twoshot": ({"COMMUX_NVLS": "0", "COMMUX_ALGO": "twoshot"}, "coll_oneshot==0,coll_twoshot>0"),
    # a 1 MiB workspace: every two-shot reduction and broadcast runs through
    # dozens of double-buffered chunks (pipeline fill, steady state, drain)
    "pipeline": ({"COMMUX_NVLS": "0", "COMMUX_CUDA_WS_BYTES": "1048576"}, "coll_twoshot>0"),
    # the opt-in chain (broadcast and large reduce along a chain of the
    # ranks), through many chunks; at 2 ranks it is not selected
    "chain": ({"COMMUX_NVLS": "0", "COMMUX_CUDA_WS_BYTES": "1048576", "COMMUX_CHAIN_RANKS": "3"}, "coll_calls>0"),
}


@pytest.mark.parametrize("variant", sorted(COLL_VARIANTS))
def test_collective_numerics_cuda(variant):
    # every rank on its own GPU (up to 8): the device kernels of the variant
    world = max(2, min(ngpu(), 8))
    extra, expect = COLL_VARIANTS[variant]
    if variant == "chain" and world >= 3:
        expect += ",coll_chain>0"
    env = topology("peer", world, (PEER_COLL + "," + expect + ",coll_gather>0", None))
    check(run("gpu_coll_numerics.py", world, env=dict(env, **extra), timeout=600))


def test_collective_numerics_cuda_shared_gpu():
    env = topology("shared", 2, (None, SHARED_COLL))
    check(run("gpu_coll_numerics.py", 2, env=dict(env, CMX_SIZES="7,70001,1048576"), timeout=600))


def test_device_barrier_orders_device_work():
    # peer GPUs only: on a shared GPU the barrier runs on the host
    env = topology("peer", 2, ("coll_barriers>0,coll_shared_gpu==0", None))
    world = max(2, min(ngpu(), 8))
    check(run("gpu_barrier.py", world, env=dict(env, CMX_BARRIER_MODE="order"), timeout=300))


def test_device_barrier_times_out_without_peer():
    # rank 1 never joins: rank 0's bounded wait runs out (1 s), the kernel
    # records it and returns, the call raises; plain peer loads, no NVLS
    env = topology("peer", 2, ("coll_shared_gpu==0", None))
    env.update(CMX_BARRIER_MODE="timeout", COMMUX_DEVICE_TIMEOUT_MS="1000", COMMUX_NVLS="0",
               NCCL_NVLS_ENABLE="0")
    check(run("gpu_barrier.py", 2, env=env, timeout=180))


def test_smoke_entry():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "__graft_entry__.py")], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


def test_plan_self():
    check(run("gpu_plan.py", 1, env=dict(CUDA, CMX_EXPECT="cuda_plan_starts>0,cuda_plan_device_msgs==0")))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_plan_two_ranks(mode):
    check(run("gpu_plan.py", 2, env=topology(mode, 2, (PEER_PLAN, SHARED_PLAN)), timeout=180))


def test_halo_cuda_batch_path_one_rank():
    check(run("halo.py", 1, env=dict(CUDA, COMMUX_HALO_PLAN="0", COMMUX_GROUP="1",
                                     CMX_EXPECT="cuda_plan_starts==0,cuda_pulls>0"), timeout=180))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_halo_cuda_batch_path(mode):
    env = topology(mode, 2, (PEER_P2P + ",cuda_plan_starts==0", SHARED_P2P + ",cuda_plan_starts==0"))
    check(run("halo.py", 2, env=dict(env, COMMUX_HALO_PLAN="0", COMMUX_GROUP="1"), timeout=180))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_ipc_mappings_bounded_under_allocator_churn(mode):
    # either way the receiver maps the sender's segments through CUDA IPC
    env = topology(mode, 2, ("cuda_pulls_peer_gpu>0,cuda_pulls_same_gpu==0", "cuda_pulls_same_gpu>0"))
    check(run("gpu_ipc_churn.py", 2, env=env, timeout=240))


@pytest.mark.parametrize("mode", ["peer", "shared"])
def test_unexportable_memory_staged(mode):
    # the caching allocator's expandable segments cannot be exported through
    # CUDA IPC: sends to another process travel through the export pool
    alloc = {"PYTORCH_CUDA_ALLOC_CONF": "expandable_segments:True"}
    env = dict(topology(mode, 2, (PEER_P2P, SHARED_P2P)), **alloc)
    check(run("gpu_p2p.py", 2, env=dict(env, CMX_EXPECT_EXPORT_STAGING="1"), timeout=240))
    env = dict(topology(mode, 2, (PEER_PLAN, SHARED_PLAN)), **alloc)
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
