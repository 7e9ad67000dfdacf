"""Shared parity arithmetic of the GPU tests (imported by the test modules; not a test).

Errors are relative L2 norms per parameter tensor. The yardstick is the oracle evaluated in
float64 (the same operations and operand roundings, exact products, accurate sums); a float32
evaluation of the oracle is carried along to measure how far plain float32 arithmetic of the
same algorithm already is from it.

fp32-class arithmetic (fp32 CUDA cores, split-bf16 tensor-core products) is held to the
gradients 1e-4, parameters after an update 1e-3. bf16 GEMM operands are
held to BF16_NOISE times the float32 oracle's own distance from the float64 oracle (floors
1e-4 and 1e-3): a layer output within float32 rounding of a bf16 rounding boundary rounds to
either neighbour depending on the summation order, and Adam's first steps (lr * sign(g) for a
fresh moment) turn a gradient element that such flips move across zero into a full step the
other way; any float32-accumulating implementation of the arithmetic shows that noise. The
tensor cores accumulate less precisely than a CPU BLAS (measured on B200: a 512-long chain of
products is ~4x further from exact than numpy's float32 product, and cuBLAS's bf16 GEMM gives
the same values as this library's for chains up to 8,192), and a ReLU or max turns those
differences into derivative flips, so for bf16 gradients the noise is also measured through
cuBLAS (tests/_cublas_ref.py) and the bound uses the larger of the two.
"""
import numpy as np

GRAD_RTOL = 1e-4
PARAM_RTOL = 1e-3
# bound on the relative change of an update per tensor: fp32 CUDA cores, split-bf16 products
# (~1e-5 relative per product, amplified by Adam's per-element normalisation), and the floor
# of the bf16 bound
CHANGE_RTOL = {"fp32": 1e-3, "bf16x3": 2e-2}
BF16_NOISE = 3.0


def rel(a, b, floor=0.0):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), floor, 1e-30))


def check_grads(tag, precision, got, truth, plain, hw=None):
    """got / truth / plain: {name: gradient} of the CUDA path, the float64 oracle and the
    float32 oracle; hw (bf16 only): the same gradient through cuBLAS bf16 GEMMs with fp32
    accumulation (tests/_cublas_ref.py), the other measure of the arithmetic's own noise.
    Returns the tensors over their bound (empty when all pass)."""
    bad = []
    for k in truth:
        e, e32 = rel(got[k], truth[k]), rel(plain[k], truth[k])
        ehw = rel(hw[k], truth[k]) if hw is not None else 0.0
        bound = (GRAD_RTOL if precision != "bf16"
                 else max(BF16_NOISE * max(e32, ehw), GRAD_RTOL))
        extra = f", cuBLAS bf16 {ehw:.3e}" if hw is not None else ""
        print(f"{tag} gradient {k}: native {e:.3e}, fp32 oracle {e32:.3e}{extra}, "
              f"bound {bound:.1e}")
        if e > bound:
            bad.append((k, e, bound))
    return bad


def check_params(tag, precision, before, got, truth, plain, steps, lr):
    """Parameters after an update: got / truth / plain as in check_grads, `before` the
    parameters the update started from. Two measures per tensor:
      * the parameters themselves (the north-star measure), relative to the float64 result; a
        tensor that starts at zero (biases) is measured against the largest move Adam can make
        in `steps` steps (steps * lr per element);
      * the change the update made, relative to the float64 oracle's change. An update that
        changed nothing has error 1 here, so this measure rejects a no-op for every tensor.
        Adam divides each gradient element by its own running magnitude, so elements whose
        gradient is within the arithmetic's rounding of zero take steps of either sign: the
        change is held to CHANGE_RTOL[precision] (fp32-class) or to BF16_NOISE times the float32
        oracle's own change error (bf16)."""
    bad = []
    for k in truth:
        floor = steps * lr * np.sqrt(truth[k].size) if not np.any(before[k]) else 0.0
        e = rel(got[k], truth[k], floor)
        e32 = rel(plain[k], truth[k], floor)
        b64 = np.asarray(before[k], np.float64)
        d_true = np.asarray(truth[k], np.float64) - b64
        c = rel(np.asarray(got[k], np.float64) - b64, d_true)
        c32 = rel(np.asarray(plain[k], np.float64) - b64, d_true)
        if precision == "bf16":
            bound = max(BF16_NOISE * e32, PARAM_RTOL)
            cbound = max(BF16_NOISE * c32, CHANGE_RTOL["bf16x3"])
        else:
            bound, cbound = PARAM_RTOL, CHANGE_RTOL[precision]
        print(f"{tag} params {k}: native {e:.3e} (fp32 oracle {e32:.3e}, bound {bound:.1e}); "
              f"change {c:.3e} (fp32 oracle {c32:.3e}, bound {cbound:.1e})")
        assert cbound < 1.0, (k, "the change bound would pass an update that changed nothing")
        if e > bound or c > cbound:
            bad.append((k, e, bound, c, cbound))
    return bad
