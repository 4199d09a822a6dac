"""API validation that happens before any device work: same exceptions and
messages as the reference (golden_meta.json 'messages')."""

import numpy as np
import pytest

import ozaki_jax_b200 as oz


def test_error_messages_match_reference(golden):
    _, meta = golden
    msgs = meta["messages"]
    cases = {
        "bad_precision": (dict(pipeline="ondevice", precision="invalid"), np.ones((2, 2)), np.ones((2, 2))),
        "bad_tuple": (dict(pipeline="ondevice", precision=(0, 1)), np.ones((2, 2)), np.ones((2, 2))),
        "bad_accumulation": (dict(pipeline="ondevice", accumulation="x"), np.ones((2, 2)), np.ones((2, 2))),
        "bad_pipeline": (dict(pipeline="gpu"), np.ones((2, 2)), np.ones((2, 2))),
        "bad_safe_mode": (dict(pipeline="ondevice", safe_mode="ignore"), np.ones((2, 2)), np.ones((2, 2))),
        "bad_shapes": (dict(pipeline="ondevice"), np.ones((2, 3)), np.ones((2, 2))),
        "bad_rank": (dict(pipeline="ondevice"), np.ones(3), np.ones((3, 2))),
    }
    for label, (kw, A, B) in cases.items():
        with pytest.raises(ValueError) as ei:
            oz.matmul(A, B, **kw)
        assert str(ei.value) == msgs[label], label


def test_mixed_families_rejected():
    import torch
    with pytest.raises(ValueError, match="both be numpy arrays"):
        oz.matmul(torch.ones(2, 2, dtype=torch.float64), np.ones((2, 2)), pipeline="ondevice")


def test_gram_residual_validation():
    rng = np.random.RandomState(0)
    with pytest.raises(ValueError, match="A must be 2D"):
        oz.gram(rng.randn(10), mode="ozaki")
    with pytest.raises(ValueError, match="mode="):
        oz.gram(rng.randn(4, 4), mode="invalid")
    with pytest.raises(ValueError, match="accumulation="):
        oz.gram(rng.randn(4, 4), mode="ozaki", accumulation="host")
    with pytest.raises(ValueError, match="x length 5 != A columns 4"):
        oz.residual(rng.randn(3, 4), rng.randn(5), rng.randn(3), mode="ozaki")
    with pytest.raises(ValueError, match="incompatible"):
        oz.residual(rng.randn(3, 4), rng.randn(4), rng.randn(4), mode="ozaki")
    with pytest.raises(ValueError, match="x must be 1D or 2D"):
        oz.residual(rng.randn(3, 4), rng.randn(4, 1, 1), rng.randn(3), mode="ozaki")


def test_gram_residual_messages_match_reference(golden):
    """Every argument check of gram / residual raises the reference's exact text
    (the reference's own messages, recorded by make_golden.py)."""
    _, meta = golden
    msgs = meta["messages"]
    one = np.ones
    cases = {
        "gram_bad_mode": (oz.gram, (one((4, 4)),), dict(mode="invalid")),
        "gram_bad_accumulation": (oz.gram, (one((4, 4)),), dict(mode="ozaki", accumulation="host")),
        "gram_not_2d": (oz.gram, (one(4),), dict(mode="ozaki")),
        "residual_bad_mode": (oz.residual, (one((3, 4)), one(4), one(3)), dict(mode="invalid")),
        "residual_bad_accumulation": (oz.residual, (one((3, 4)), one(4), one(3)),
                                      dict(mode="ozaki", accumulation="host")),
        "residual_not_2d": (oz.residual, (one(4), one(4), one(4)), dict(mode="ozaki")),
        "residual_x_length": (oz.residual, (one((3, 4)), one(5), one(3)), dict(mode="ozaki")),
        "residual_b_vector": (oz.residual, (one((3, 4)), one(4), one(4)), dict(mode="ozaki")),
        "residual_x_rows": (oz.residual, (one((3, 4)), one((5, 2)), one((3, 2))), dict(mode="ozaki")),
        "residual_b_matrix": (oz.residual, (one((3, 4)), one((4, 2)), one((3, 3))), dict(mode="ozaki")),
        "residual_x_ndim": (oz.residual, (one((3, 4)), one((4, 1, 1)), one(3)), dict(mode="ozaki")),
    }
    for label, (fn, args, kw) in cases.items():
        assert msgs[label], label
        with pytest.raises(ValueError) as ei:
            fn(*args, **kw)
        assert str(ei.value) == msgs[label], label


def test_preflight_bound_reasons():
    from ozaki_jax_b200.matmul import _bound_reasons
    from ozaki_jax_b200.host import host_safety_reasons
    # FP32 extraction stays within the bound up to K = 2^22; beyond, bits <= 0
    for K in (1, 64, 1024, 8192, 65536, 2 ** 20, 2 ** 22):
        assert _bound_reasons(K, 24 - oz.compute_rho_f32(K), "x") == []
    assert _bound_reasons(2 ** 22 + 1, 24 - oz.compute_rho_f32(2 ** 22 + 1), "x")
    # host pipeline: K=10000 with 8 slices is unsafe (ci_cpu_validate.py:108-111)
    rho, reasons = host_safety_reasons(10000, 8)
    assert reasons == ["insufficient slice budget: n_slices*bits_per_slice=40 < 53"]


def test_accumulate_2sum_backend_text_without_gpu():
    """The reference's backend error text, raised before any device work."""
    import numpy as np
    import ozaki_jax_b200 as oz
    with pytest.raises(ValueError) as ei:
        oz.accumulate_2sum(np.zeros((1, 2, 2), np.float32), np.ones((1, 2), np.float32),
                           np.ones((1, 2), np.float32), ((1,),), backend="xla")
    assert str(ei.value) == "Unknown backend='xla'; expected 'auto', 'jax', or 'pallas'."


def test_public_names_match_the_reference_hot_path():
    import ozaki_jax_b200 as oz
    for name in ("matmul", "matmul_numpy", "gram", "residual", "extract_split_rows",
                 "extract_split_cols", "f32_extract_split_rows", "f32_extract_split_cols",
                 "jax_extract_split_rows", "jax_extract_split_cols", "accumulate_2sum",
                 "validate_accumulation_2sum"):
        assert callable(getattr(oz, name)), name


def test_no_cpu_fallback_without_a_device():
    """With no CUDA device the product path raises instead of computing on the
    host: valid calls of every public compute function fail loudly."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is visible")
    A = np.ones((8, 8))
    calls = [lambda: oz.matmul(A, A, pipeline="ondevice"),
             lambda: oz.matmul(A, A, pipeline="host"),
             lambda: oz.gram(A, mode="ozaki"),
             lambda: oz.residual(A, np.ones(8), np.ones(8), mode="ozaki")]
    for call in calls:
        with pytest.raises(RuntimeError, match="needs a CUDA device"):
            call()
