"""Host-side logic of the Python layer that needs no GPU."""
import fp4_gemm


def test_forward_host_chunk_schedule():
    for m in (1, 60, 127, 128, 129, 700, 2048, 4096, 5000):
        for chunk in (128, 256, 512):
            sizes = fp4_gemm._chunk_schedule(m, chunk)
            assert sum(sizes) == m
            assert all(0 < s <= chunk for s in sizes)
            assert all(s == chunk for s in sizes[:-1])
    assert fp4_gemm._chunk_schedule(2048, 512) == [512] * 4
    assert fp4_gemm._chunk_schedule(700, 256) == [256, 256, 188]
