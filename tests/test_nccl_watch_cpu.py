"""NCCL failure detection, host side (no GPU): the bounded polling in rt/nccl_watch.hpp that the
library runs around every collective, driven by fakes of the stream and of the communicator.

A rank that left shows up either as an NCCL error reported by ncclCommGetAsyncError (its peers'
connections closed) or as silence (the collective never completes); both must end the wait with
OVVS_STATUS_ERROR and ask for the communicator to be aborted, the second at the deadline. The
reference fails closed in the same way (src/prim/mixer.cpp:47-50)."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

HARNESS = r"""
#include <cstdio>
#include <vector>
#include "rt/nccl_watch.hpp"
using namespace ovvs::rt;

struct Clock { long long t = 0; long long operator()() const { return t; } };

int main() {
  // settle_nccl
  {
    Clock c; auto pause = [&] { c.t += 10; };
    auto never = [](ncclResult_t* s) { *s = ncclInProgress; return ncclSuccess; };
    WatchResult w = settle_nccl(ncclSuccess, never, [&] { return c.t; }, pause, 100);
    std::printf("settle_success %d %d\n", w.status, w.abort);
    int polls = 0;
    auto later = [&](ncclResult_t* s) { *s = ++polls < 3 ? ncclInProgress : ncclSuccess; return ncclSuccess; };
    w = settle_nccl(ncclInProgress, later, [&] { return c.t; }, pause, 100);
    std::printf("settle_progress_then_ok %d %d %d\n", w.status, w.abort, polls);
    auto remote = [](ncclResult_t* s) { *s = ncclRemoteError; return ncclSuccess; };
    w = settle_nccl(ncclInProgress, remote, [&] { return c.t; }, pause, 100);
    std::printf("settle_remote_error %d %d\n", w.status, w.abort);
    w = settle_nccl(ncclSystemError, never, [&] { return c.t; }, pause, 100);
    std::printf("settle_call_failed %d %d\n", w.status, w.abort);
    c.t = 0;
    w = settle_nccl(ncclInProgress, never, [&] { return c.t; }, pause, 100);
    std::printf("settle_deadline %d %d %lld\n", w.status, w.abort, c.t);
  }
  // watch_stream
  {
    Clock c; auto pause = [&] { c.t += 10; };
    auto ok = [](ncclResult_t* s) { *s = ncclSuccess; return ncclSuccess; };
    int q = 0;
    auto busy3 = [&] { return ++q <= 3 ? StreamState::kBusy : StreamState::kIdle; };
    WatchResult w = watch_stream(busy3, ok, [&] { return c.t; }, pause, 1000);
    std::printf("watch_done %d %d %d\n", w.status, w.abort, q);
    auto busy = [] { return StreamState::kBusy; };
    int polls = 0;
    auto peer_left = [&](ncclResult_t* s) { *s = ++polls < 5 ? ncclSuccess : ncclRemoteError; return ncclSuccess; };
    c.t = 0;
    w = watch_stream(busy, peer_left, [&] { return c.t; }, pause, 100000);
    std::printf("watch_peer_reported %d %d %d\n", w.status, w.abort, polls);
    c.t = 0;
    w = watch_stream(busy, ok, [&] { return c.t; }, pause, 500);
    std::printf("watch_peer_silent %d %d %lld\n", w.status, w.abort, c.t);
    auto failed = [] { return StreamState::kFailed; };
    w = watch_stream(failed, ok, [&] { return c.t; }, pause, 500);
    std::printf("watch_stream_failed %d %d\n", w.status, w.abort);
  }
  return 0;
}
"""


def test_nccl_watch_logic(tmp_path):
    cxx = shutil.which("g++")
    cuda_inc = "/usr/local/cuda/include"
    if not cxx or not os.path.exists(os.path.join(cuda_inc, "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    src = tmp_path / "watch.cpp"
    src.write_text(HARNESS)
    exe = tmp_path / "watch"
    subprocess.run([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "ovvs_b200", "csrc"),
                    "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    res = {line.split()[0]: [int(v) for v in line.split()[1:]] for line in out.splitlines()}
    OK, ERR = 0, 1  # OVVS_STATUS_SUCCESS, OVVS_STATUS_ERROR
    assert res["settle_success"] == [OK, 0]
    assert res["settle_progress_then_ok"] == [OK, 0, 3]
    assert res["settle_remote_error"] == [ERR, 1]
    assert res["settle_call_failed"] == [ERR, 1]
    status, abort, t = res["settle_deadline"]
    assert (status, abort) == (ERR, 1) and 100 < t <= 120
    assert res["watch_done"] == [OK, 0, 4]
    assert res["watch_peer_reported"] == [ERR, 1, 5]  # the rank that left is reported by NCCL
    status, abort, t = res["watch_peer_silent"]
    assert (status, abort) == (ERR, 1) and 500 < t <= 520  # nothing reported: the deadline
    assert res["watch_stream_failed"] == [ERR, 0]
