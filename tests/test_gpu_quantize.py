"""The load-time encoders on the GPU give the host encoders' bytes
(lrs_quantize_matrix_device vs lrs_quantize_matrix), for every type,
including the reference encoders' fallbacks (cols not a multiple of 256)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TYPES = ["Q4_K", "Q6_K", "Q5_0", "Q8_0", "Q4_0", "Q4_1", "Q5_1", "Q5_K", "F16", "BF16"]


@pytest.mark.parametrize("shape", [(48, 512), (17, 896)], ids=str)
@pytest.mark.parametrize("qt", TYPES)
def test_device_encoders_match_host(lrs, backend, qt, shape):
    import torch
    rows, cols = shape
    rng = np.random.default_rng(3)
    v = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    v[1] = 0.0                      # an all-zero row
    v[2, :64] = 1e-20               # tiny values
    v[3, ::7] *= 300.0              # outliers
    host = lrs.QuantTensor.quantize(v.ravel(), rows, cols, lrs.QuantType[qt])
    dv = torch.from_numpy(v).cuda()
    out = torch.zeros(host.data.size + 16, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()  # the encoder runs on the backend's own stream
    t, n = backend.quantize_device(dv.data_ptr(), rows, cols, lrs.QuantType[qt], out.data_ptr(),
                                   out.numel())
    assert t == host.quant_type and n == host.data.size
    got = out[:n].cpu().numpy()
    assert np.array_equal(got, host.data), f"{int((got != host.data).sum())} bytes differ"
