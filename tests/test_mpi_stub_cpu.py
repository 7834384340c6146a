"""The multi-process MPI stand-in that lets the reference driver run as several
ranks in an image without MPI (oracle/mpi_stub_tcp/mpi.h): its self-test,
compiled here and run as 1 to 8 processes with the environment torchrun
gives (RANK, WORLD_SIZE, MASTER_ADDR), checks communicator splits, tagged
point-to-point messages (large, and matched out of order), broadcasts,
reductions, gathers and barriers; and a rank that exits early makes the
others fail instead of hanging."""
import os
import socket
import subprocess

import pytest

from conftest import ROOT

STUB = os.path.join(ROOT, "oracle", "mpi_stub_tcp")


@pytest.fixture(scope="module")
def selftest(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("mpi_stub") / "selftest")
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", STUB, "-o", out, os.path.join(STUB, "selftest.cpp"),
                    "-lpthread"], check=True)
    return out


def free_base(n):
    """A base port with n free consecutive ports."""
    for _ in range(50):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        base = s.getsockname()[1]
        s.close()
        if base + n >= 65535:
            continue
        ok = True
        for p in range(base, base + n):
            t = socket.socket()
            try:
                t.bind(("127.0.0.1", p))
            except OSError:
                ok = False
            finally:
                t.close()
        if ok:
            return base
    raise RuntimeError("no free port range")


def launch(binary, world, extra_env=None):
    """Runs world ranks; a run in which a rank could not bind its port (taken
    by another process between the check and the bind) is retried on a new
    port range, up to three times."""
    for attempt in range(3):
        outs = launch_once(binary, world, extra_env)
        if not any("bind to port" in e for _, _, e in outs):
            break
    return outs


def launch_once(binary, world, extra_env=None):
    base = free_base(world)
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   ABFT_MPI_STUB_PORT=str(base), ABFT_MPI_STUB_TIMEOUT="30")
        env.update((extra_env or {}).get(r, {}))
        procs.append(subprocess.Popen([binary], env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                      text=True))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o, e))
    return outs


@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_selftest_all_world_sizes(selftest, world):
    outs = launch(selftest, world)
    for r, (rc, o, e) in enumerate(outs):
        assert rc == 0, (r, o, e)
        assert o.strip() == f"ok {r}", (r, o, e)


def test_rank_that_dies_does_not_hang_the_others(selftest):
    # rank 1 gets a WORLD_SIZE it cannot satisfy and exits at once; the
    # others must end with an error (its connection never comes or closes)
    short = {"ABFT_MPI_STUB_TIMEOUT": "5"}
    outs = launch(selftest, 3, extra_env={0: short, 1: dict(short, RANK="7"), 2: short})
    assert outs[1][0] != 0
    assert any(rc != 0 for rc, _, _ in (outs[0], outs[2]))
    for rc, o, e in outs:
        assert "ok" not in o or rc == 0
