"""The measurement probes the bench's rooflines come from, on a B200.

mapal_gpu_probe_mma_peak issues the 3xTF32 GEMM's own tcgen05.mma shape
with operands resident in shared memory; its rates must sit in a band around
the B200's dense figures (tf32 1125, bf16 2250 TFLOP/s nominal; the probe
reads about 1000-1100 and 1950-1980 at full clock), with bf16 about twice
tf32 (K16 against K8 per instruction) and the MN-major B form near the
K-major one. The band's floors leave room for a GPU held below its top clock.
mapal_gpu_probe_launch_floor's read floor must stream its input (a 64 MiB
read takes at least 64 MiB / twice the measured copy rate), and both probes
reject bad arguments with an error instead of launching."""
import pytest
import torch

import flow_b200 as fb

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def test_mma_probe_rates(ctx):
    tf32 = max(ctx.probe_mma_peak(0, 1024) for _ in range(2))
    bf16 = max(ctx.probe_mma_peak(1, 1024) for _ in range(2))
    tf32_mn = max(ctx.probe_mma_peak(2, 1024) for _ in range(2))
    assert 300.0 < tf32 < 1300.0, tf32
    assert 600.0 < bf16 < 2600.0, bf16
    assert 1.4 < bf16 / tf32 < 2.6, (bf16, tf32)
    assert 0.5 * tf32 < tf32_mn < 1.3 * tf32, (tf32_mn, tf32)


def test_mma_probe_rejects_bad_arguments(ctx):
    with pytest.raises(fb.MapalInfraError):
        ctx.probe_mma_peak(3, 64)
    with pytest.raises(fb.MapalInfraError):
        ctx.probe_mma_peak(0, 0)
    # the context stays usable
    assert ctx.probe_mma_peak(0, 64) > 0.0


def _time_ms(fn, reps=5):
    s = torch.cuda.current_stream()
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def test_launch_floors_run_and_read_floor_streams(ctx):
    n = 1 << 24  # 64 MiB of floats
    x = torch.ones(n, dtype=torch.float32, device="cuda")
    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    empty_ms = _time_ms(lambda: ctx.probe_launch_floor(0))
    read_ms = _time_ms(lambda: ctx.probe_launch_floor(1, x, sink))
    ctx.probe_launch_floor(2, x, sink)
    ctx.synchronize()
    assert empty_ms < 0.05, empty_ms
    # 64 MiB at twice a B200's ~6.6 TB/s copy rate is 10 us; a read that
    # skipped its loads would finish near the empty kernel's time
    assert read_ms > 4 * n / 13.0e12 * 1e3, read_ms
    assert read_ms < 1.0, read_ms


def test_launch_floor_rejects_bad_arguments(ctx):
    x = torch.ones(6, dtype=torch.float32, device="cuda")
    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    with pytest.raises(fb.MapalInfraError):
        ctx.probe_launch_floor(1, x, sink)  # not a multiple of 4 floats
    with pytest.raises(fb.MapalInfraError):
        ctx.probe_launch_floor(2, None, sink)
    with pytest.raises(fb.MapalInfraError):
        ctx.probe_launch_floor(7)
