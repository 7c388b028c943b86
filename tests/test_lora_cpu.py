"""Low-rank adapters without a GPU: the oracle's restatement of the
reference's fold and delta, and the C-ABI's refusals of null arguments."""
import numpy as np

from oracle import lib, lora_np


def test_scale_fold_is_one_rounding():
    rng = np.random.default_rng(5)
    a = lib.f32_to_bf16(rng.standard_normal((7, 64)).astype(np.float32))
    # x1 is the identity; x2 and x0.5 are exact (exponent shifts)
    assert np.array_equal(lora_np.fold_scale(a, 1.0), a)
    af = lib.bf16_to_f32(a)
    assert np.array_equal(lib.bf16_to_f32(lora_np.fold_scale(a, 2.0)), af * 2)
    assert np.array_equal(lib.bf16_to_f32(lora_np.fold_scale(a, 0.5)), af * 0.5)
    # a general factor: the f32 product rounded once to bf16
    got = lib.bf16_to_f32(lora_np.fold_scale(a, 0.37))
    want = lib.bf16_to_f32(lib.f32_to_bf16((af * np.float32(0.37)).astype(np.float32)))
    assert np.array_equal(got, want)


def test_runtime_delta_equals_folded_weight():
    """x (W + B A)^T == x W^T + (x A^T) B^T: the identity the reference's
    block test rests on (tests/ltx25-lora-apply-test.cc:357-370, 418-440)."""
    rng = np.random.default_rng(6)
    M, K, N, r = 9, 64, 48, 5
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    a = rng.standard_normal((r, K)).astype(np.float32)
    b = rng.standard_normal((N, r)).astype(np.float32)
    folded = x.astype(np.float64) @ lora_np.fold(w, a, b).astype(np.float64).T
    runtime = x.astype(np.float64) @ w.astype(np.float64).T + lora_np.delta(x, a, b)
    assert np.abs(folded - runtime).max() < 1e-4 * np.abs(runtime).max()


def test_adapter_abi_refuses_nulls_without_a_device():
    import ltx25_b200 as L
    lib_ = L.load()
    assert lib_.ltx_lora_upload(None, None, None, 4, 64, 64, 1.0, 0, None) == -1
    assert lib_.ltx_lora_add(None, None, None, 64, None, 64, 1, 64, 64, None) == -1
    assert lib_.ltx_qlinear_lora(None, None, None, None, 64, None, None, 64, 1, 64, 64, 0,
                                 None, None) == -1
    assert lib_.ltx_block_set_lora(None, b"attn1.to_q", None) == -1
    assert lib_.ltx_lora_info(None, None, None, None) == -1
    lib_.ltx_lora_free(None)
