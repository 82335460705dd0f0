"""Descriptor exchange between ranks (rt/fd_exchange.hpp), host side, no GPU.

Sharded searches share each query's bound between ranks through GPU memory that every rank
exports as a POSIX file descriptor and every peer imports. The exchange of those descriptors is
plain host code: here N forked processes each offer a memfd holding their rank and must receive
every peer's (reading the peer's rank through it); a rank that never appears must end the
exchange with a failure at the deadline instead of a hang."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

HARNESS = r"""
#include <sys/mman.h>
#include <sys/wait.h>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "rt/fd_exchange.hpp"
using namespace ovvs::rt;

// Child `rank` of `world` (ranks listed in `skip` never start): prints one line.
static int child(uint64_t tag, int rank, int world, int64_t timeout_ms) {
  int fd = memfd_create("ovvs-test", 0);
  if (fd < 0 || ftruncate(fd, 4) != 0) return 2;
  int32_t me = 1000 + rank;
  if (pwrite(fd, &me, 4, 0) != 4) return 2;
  std::vector<int> peer;
  const int64_t t0 = fdx_now_ms();
  const bool ok = exchange_fds(tag, rank, world, fd, peer, timeout_ms);
  const int64_t dt = fdx_now_ms() - t0;
  int good = 0;
  for (int p = 0; p < world; ++p) {
    if (p == rank || peer[p] < 0) continue;
    int32_t v = 0;
    if (pread(peer[p], &v, 4, 0) == 4 && v == 1000 + p) ++good;
    close(peer[p]);
  }
  std::printf("rank %d ok %d good %d ms %lld\n", rank, ok ? 1 : 0, good, (long long)dt);
  std::fflush(stdout);
  return 0;
}

int main(int argc, char** argv) {
  const int world = std::atoi(argv[1]);
  const int absent = std::atoi(argv[2]);  // rank that never starts, or -1
  const int64_t timeout_ms = std::atoll(argv[3]);
  const uint64_t tag = 0x5eed0000ull + static_cast<uint64_t>(getpid());
  std::vector<pid_t> kids;
  for (int r = 0; r < world; ++r) {
    if (r == absent) continue;
    pid_t pid = fork();
    if (pid == 0) _exit(child(tag, r, world, timeout_ms));
    kids.push_back(pid);
  }
  int rc = 0;
  for (pid_t k : kids) {
    int st = 0;
    waitpid(k, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) rc = 1;
  }
  return rc;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("needs g++")
    d = tmp_path_factory.mktemp("fdx")
    src = d / "fdx.cpp"
    src.write_text(HARNESS)
    exe = d / "fdx"
    subprocess.run([cxx, "-std=c++17", "-O1", "-pthread", "-I",
                    os.path.join(ROOT, "ovvs_b200", "csrc"), str(src), "-o", str(exe)], check=True)
    return str(exe)


def _run(exe, world, absent, timeout_ms):
    out = subprocess.run([exe, str(world), str(absent), str(timeout_ms)], check=True,
                         capture_output=True, text=True, timeout=60).stdout
    res = {}
    for line in out.splitlines():
        f = line.split()
        res[int(f[1])] = dict(ok=int(f[3]), good=int(f[5]), ms=int(f[7]))
    return res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_every_rank_gets_every_peer(harness, world):
    res = _run(harness, world, -1, 20000)
    assert sorted(res) == list(range(world))
    for r in range(world):
        assert res[r]["ok"] == 1 and res[r]["good"] == world - 1, res


def test_absent_rank_fails_at_the_deadline(harness):
    res = _run(harness, 3, 2, 1500)
    assert sorted(res) == [0, 1]
    for r in (0, 1):
        assert res[r]["ok"] == 0, res           # failure, reported ...
        assert 1400 <= res[r]["ms"] <= 6000, res  # ... at the deadline, not a hang
