"""The allocation-free search entry point (ovvsBruteForceSearchDeviceNoAlloc).

It is meant for callers that cannot let the library allocate GPU memory -- for example when
another allocator already holds the device's free memory, or in a latency-critical loop where a
cudaMalloc/cudaFree (and the device synchronisation it implies) is not acceptable. Its results
must equal the regular device search's, call after call, although every call reuses the same
fixed scratch array. This file is collected last so that a failure here stops a `-x` run only
after every other test has run; it also passes alone in a fresh process.
"""

import numpy as np
import pytest

from tests.helpers import assert_search_close

pytestmark = pytest.mark.gpu


def _device_arrays(torch, q, nq, k):
    dq = torch.from_numpy(q).cuda()
    dn = torch.full((nq, k), -7, dtype=torch.int64, device="cuda")
    dd = torch.full((nq, k), 7.0, dtype=torch.float32, device="cuda")
    return dq, dn, dd


@pytest.mark.parametrize("metric,dtype", [("l2", "f16"), ("inner_product", "f32"),
                                          ("cosine", "f32")])
def test_no_alloc_matches_regular_search_twice(metric, dtype, ovvs, gpu, oracle):
    import torch

    rng = np.random.default_rng(2024)
    data = rng.standard_normal((30000, 96)).astype(np.float32)
    if dtype == "f16":
        data = data.astype(np.float16)
    q = rng.standard_normal((1000, 96)).astype(np.float32)
    k = 10
    ix = ovvs.BruteIndex.build(data, metric=metric, dtype=dtype, resources=gpu)
    dq, ref_n, ref_d = _device_arrays(torch, q, 1000, k)
    torch.cuda.synchronize()
    ix.search_device(dq, k, ref_n, ref_d)
    gpu.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    outs = [_device_arrays(torch, q, 1000, k)[1:] for _ in range(2)]
    torch.cuda.synchronize()
    free = []
    for call, (got_n, got_d) in enumerate(outs):  # the array keeps the previous call's contents
        ix.search_device_no_alloc(dq, k, got_n, got_d, stream=stream)
        free.append(torch.cuda.mem_get_info()[0])
        assert torch.equal(got_n, ref_n), f"ids differ on call {call}"
        # same kernels and inputs: the distances are bit-identical, within any tolerance
        assert np.array_equal(got_d.cpu().numpy().view(np.uint32),
                              ref_d.cpu().numpy().view(np.uint32)), f"distances on call {call}"
    # the first call on the device may load the array; later calls take no device memory at all
    assert free[1] == free[0], f"free device memory changed by {free[0] - free[1]} bytes"
    ix.close()
    # and the results are the reference's (the CPU oracle: ids equal, distances bit-identical
    # but for near-ties at the k-th distance within the parity tolerance)
    data32 = data.astype(np.float32)
    rnb, rds = oracle.brute_search(data32, q, k, metric)

    def exact(qi, rid):
        v = oracle.pairwise(metric, q[qi:qi + 1], data32[rid:rid + 1])[0, 0]
        return -v if metric == "inner_product" else v

    assert_search_close(outs[1][0].cpu().numpy(), outs[1][1].cpu().numpy(), rnb, rds, k, exact,
                        2e-3 if dtype == "f16" else 1e-4, what=f"no-alloc {metric}/{dtype}",
                        atol_floor=1.0)


def test_no_alloc_with_bitset_and_rejects_oversize(ovvs, gpu):
    import torch

    rng = np.random.default_rng(7)
    data = rng.standard_normal((5000, 32)).astype(np.float32)
    q = rng.standard_normal((300, 32)).astype(np.float32)
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    bits = ovvs.bitset_from_allow_list(5000, np.arange(0, 5000, 3))
    dbits = torch.from_numpy(bits).cuda()
    dq, ref_n, ref_d = _device_arrays(torch, q, 300, 5)
    torch.cuda.synchronize()
    ix.search_device(dq, 5, ref_n, ref_d, bitset=dbits)
    gpu.synchronize()
    for _ in range(2):
        _, got_n, got_d = _device_arrays(torch, q, 300, 5)
        torch.cuda.synchronize()
        ix.search_device_no_alloc(dq, 5, got_n, got_d, bitset=dbits)
        assert torch.equal(got_n, ref_n)
        assert torch.equal(got_d, ref_d)
    # more queries than the fixed array holds: a clear error, nothing written
    big = torch.zeros((400_000, 32), dtype=torch.float32, device="cuda")
    out_n = torch.full((400_000, 5), -3, dtype=torch.int64, device="cuda")
    out_d = torch.zeros((400_000, 5), dtype=torch.float32, device="cuda")
    with pytest.raises(ovvs.OvvsError) as e:
        ix.search_device_no_alloc(big, 5, out_n, out_d)
    assert e.value.status == 6  # OVVS_STATUS_SHAPE_MISMATCH
    assert int(out_n.min()) == -3
    ix.close()
