"""bt_clip_adam_noalloc: the optimizer step for callers that cannot allocate device memory
where they run it (for example an XLA FFI custom call, which runs after XLA has reserved
most of the GPU for its own allocator). It must give the same result as bt_clip_adam,
which takes its scratch from the stream-ordered allocator. The file is named to be
collected last, so that a stop at its first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest


def _call(fn, p, m, v, g, n, count, opt):
    import torch

    from boonta_b200 import _lib

    _lib.check(fn(p.data_ptr(), m.data_ptr(), v.data_ptr(), g.data_ptr(), n, count, C.byref(opt),
                  torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
def test_noalloc_optimizer_step_matches_the_allocating_one_on_two_calls():
    import torch

    from boonta_b200 import _lib

    lib = _lib.lib()
    opt = _lib.OptimizerC(3e-4, 0.5, 0.9, 0.999, 1e-8, 0.0)
    rng = np.random.default_rng(7)
    n = 1_000_003
    p0 = torch.as_tensor(rng.standard_normal(n).astype(np.float32), device="cuda")
    grads = [torch.as_tensor(rng.standard_normal(n).astype(np.float32), device="cuda")
             for _ in range(2)]
    ref = [p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")]
    out = [p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")]
    for step, g in enumerate(grads):  # two calls in a row, the second reusing the scratch
        _call(lib.bt_clip_adam, *ref, g, n, step, opt)
        _call(lib.bt_clip_adam_noalloc, *out, g, n, step, opt)
        torch.cuda.synchronize()
        for a, b in zip(out, ref):
            np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=1e-5, atol=1e-7)


def test_noalloc_optimizer_step_rejects_sizes_beyond_its_scratch():
    """Checked on the host before any GPU work, so this runs without a GPU (it needs only the
    built library)."""
    from boonta_b200 import _lib

    if not _lib.LIB_PATH.exists():
        pytest.skip("the native library is not built")

    lib = _lib.lib()
    opt = _lib.OptimizerC(3e-4, 0.5, 0.9, 0.999, 1e-8, 0.0)
    fake = C.c_void_p(256)  # never dereferenced: the size check fails first
    rc = lib.bt_clip_adam_noalloc(fake, fake, fake, fake, 134_217_728 + 1, 0, C.byref(opt), None)
    assert rc == _lib.BT_ERR_INVALID
    assert b"fixed scratch limit" in lib.bt_last_error()
