"""The allocation-free entry point, rosenna_use_model_device_noalloc_f32.

Some callers cannot let the library allocate device memory while they run: a
solver that gives all free GPU memory to its own pool allocator at start-up, or
a time-step loop that cannot absorb the device-wide synchronisation of
cudaMalloc/cudaFree.  This entry point takes the plan's intermediate buffers
from a fixed 64 MiB array in device memory instead of allocating them.

Checked through the C ABI against rosenna_use_model_device_f32 on models whose
plans pass intermediates between kernels, for two calls in a row (the array
keeps the previous call's contents), within the limits of oracle/parity.py
(max abs 1e-5; max rel 1e-4 where |ref| >= 0.1); that the calls leave the
device's free memory unchanged (the array is created at initialize, not inside
the first call); and the rejection of a batch whose intermediates do not fit.
This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from oracle import parity
from rosenna_b200 import api, workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["cnn", "lstm"])
def test_noalloc_matches_device_entry_point(name, tmp_path):
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    api.set_devices([0])
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    try:
        assert len(api.plan_description().strip().splitlines()) >= 2  # intermediates between kernels
        stream = torch.cuda.current_stream().cuda_stream
        w = workloads.WORKLOADS[name]
        for call, n in enumerate((1000, 1537)):
            ins = workloads.make_inputs_torch(name, n, device="cuda", seed_offset=call)
            ref = [torch.zeros((r, n), dtype=torch.float32, device="cuda") for r in w.output_rows]
            got = [torch.full((r, n), float("nan"), dtype=torch.float32, device="cuda") for r in w.output_rows]
            ip = [x.data_ptr() for x in ins]
            api.use_model_device(n, ip, [o.data_ptr() for o in ref], stream)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            api.use_model_device_noalloc(n, ip, [o.data_ptr() for o in got], stream)
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info()[0] == free_before, f"{name} call {call}: device memory changed"
            for g, r in zip(got, ref):
                res = parity.compare(g.double().cpu().numpy(), r.double().cpu().numpy())
                print(f"{name} call {call}: {parity.describe(res)}")
                assert res["ok"], f"{name} call {call}: {parity.describe(res)}"
        # a batch whose intermediates exceed the fixed array is refused with the limit in the message
        big = 1 << 24
        with pytest.raises(api.RosennaError) as e:
            api.use_model_device_noalloc(big, ip, [o.data_ptr() for o in got], stream)
        assert e.value.code == api.ERR_SHAPE and "bytes" in str(e.value)
    finally:
        api.finalize()
