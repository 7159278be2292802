"""Host-resident GEMM with copy/compute overlap (vg_host_pipeline_gemm_f16).

Consecutive calls share the pipeline's device buffers and overlap on the GPU, so the
second call's uploads must wait for the first call's GEMMs and its GEMMs for the first
call's downloads. Each result is checked against the device-resident entry point.
"""
import numpy as np
import pytest

from conftest import to_dev, to_host

pytestmark = pytest.mark.gpu


def _pinned(a_u16):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a_u16).view(np.int16)).view(torch.float16)
    return t.pin_memory()


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_pipeline_two_calls_in_flight(vg, orc, chunks):
    import torch
    pipe = vg.HostPipeline(chunks=chunks)
    M, N, K = 1000, 1536, 640
    ins = [orc.make_inputs(M, N, K, seed_a=s, seed_b=s + 1) for s in (3, 11)]
    outs = [torch.empty((M, N), dtype=torch.float16).pin_memory() for _ in ins]
    stream = torch.cuda.current_stream()
    for (A, B), C in zip(ins, outs):
        pipe.gemm(_pinned(A), _pinned(B), C, stream=stream)
    stream.synchronize()
    for (A, B), C in zip(ins, outs):
        want = to_host(vg.gemm(to_dev(A), to_dev(B)))
        torch.cuda.synchronize()
        got = C.view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got, want)
    pipe.close()


def test_pipeline_rejects_unpinned(vg):
    import torch
    pipe = vg.HostPipeline()
    a = torch.zeros(8, 16, dtype=torch.float16)
    with pytest.raises(ValueError):
        pipe.gemm(a, a, torch.zeros(8, 8, dtype=torch.float16))
    pipe.close()
