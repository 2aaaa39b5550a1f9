"""Failure detection without a GPU fault: a pipeline wait that nothing
satisfies runs out after its limit, records its code in the device status
word and returns; the host reads the status, and the context stays usable
(a forward + backward afterwards still matches the oracle)."""

import pytest
import torch

from mlx_cce import _ext

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_reports_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.cuda.set_device(0)
    _ext.device_status(reset=True)  # clean start
    stream = torch.cuda.current_stream()
    rc = _ext.lib.cce_selftest_wait_timeout(50_000_000, stream.cuda_stream)  # 50 ms
    assert rc == _ext.CCE_OK
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="code 99"):
        _ext.device_status()
    with pytest.raises(RuntimeError, match="code 99"):
        _ext.device_status(reset=True)  # reports, then clears
    _ext.device_status()  # clear now
    assert _ext.lib.cce_selftest_wait_timeout(0, None) == _ext.CCE_ERR_ARG
    # the context still runs the real kernels correctly
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_parity_gpu import check, oracle, run, small
    e, c, t, _ = small(130, 64, 1000, torch.bfloat16, seed=21)
    check(run(e, c, t), oracle(e, c, t), torch.bfloat16)
    _ext.device_status()
