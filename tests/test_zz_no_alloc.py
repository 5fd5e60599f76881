"""jhq_search_device_noalloc: the search for callers that may not allocate
device memory while serving (a host owning a fixed memory pool, real-time
paths, a framework that reserved the GPU). Its temporaries live in a fixed
array inside the library. The results must equal jhq_search_device's bit for
bit (the tolerance every parity test here uses), on two calls in a row, since
the array keeps the previous call's contents. Collected last on purpose."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _index(jhq, d, M, nlist, nprobe, batch, n, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, d), dtype=np.float32)
    idx = jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=nlist, nprobe=nprobe, batch_size=batch))
    idx.train(x[:2000])
    idx.add(x)
    return idx, rng.standard_normal((150, d), dtype=np.float32)


@pytest.mark.parametrize("nq", [150, 20])            # more / fewer queries than one batch
@pytest.mark.parametrize("d,M,nlist,nprobe,batch", [(128, 32, 1, 1, 64), (64, 16, 16, 4, 50)])
def test_noalloc_matches_search_device_twice(jhq, d, M, nlist, nprobe, batch, nq):
    """Bit-equal to jhq_search_device on two calls in a row, and the device's free
    memory does not move across the second call (nothing is allocated)."""
    import torch
    idx, q = _index(jhq, d, M, nlist, nprobe, batch, 6000, d + nlist)
    q = q[:nq]
    k = 10
    tq = torch.from_numpy(q).cuda()
    ref_d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    ref_i = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    idx.search_device(tq.data_ptr(), nq, k, ref_d.data_ptr(), ref_i.data_ptr(), s)
    outs = [(torch.full((nq, k), -7.0, dtype=torch.float32, device="cuda"),
             torch.full((nq, k), -7, dtype=torch.int32, device="cuda")) for _ in range(2)]
    torch.cuda.synchronize()
    for call, (out_d, out_i) in enumerate(outs):
        free0 = torch.cuda.mem_get_info()[0]
        idx.search_device_noalloc(tq.data_ptr(), nq, k, out_d.data_ptr(), out_i.data_ptr(), s)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert torch.equal(out_i, ref_i), f"ids differ on call {call}"
        assert torch.equal(out_d, ref_d), f"distances differ on call {call}"
        if call == 1:                              # after the first call's one-time set-up
            assert free1 == free0, f"device memory moved by {free0 - free1} bytes"
    idx.check_device_status()


def test_noalloc_rejects_oversized_batch(jhq):
    import torch
    idx, _ = _index(jhq, 64, 16, 1024, 8, 8192, 5000, 3)
    q = np.random.default_rng(4).standard_normal((8192, 64), dtype=np.float32)
    tq = torch.from_numpy(q).cuda()                        # 8192 x 1024 coarse scores = 32 MiB
    out_d = torch.empty((len(q), 10), dtype=torch.float32, device="cuda")
    out_i = torch.empty((len(q), 10), dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        idx.search_device_noalloc(tq.data_ptr(), len(q), 10, out_d.data_ptr(), out_i.data_ptr())
