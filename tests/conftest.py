"""Shared test setup.

- registers the `gpu` marker (tests that need a B200 and the built CUDA engine);
- puts the engine's Python bindings (qwen3-tts_b200/) and the parity oracle
  (oracle/, test infrastructure) on sys.path;
- selects the reference's f32-activation kernels for the oracle process
  (QWEN_NO_BF16DOT / QWEN_NO_VNNI / QWEN_NO_SDOT = 1, the semantics the
  reference's own `make test-selftest` fallback run uses, Makefile:756-761);
- selects the reference's sequential code-predictor prefill
  (QWEN_CP_PREFILL2 = 0): positions 0 and 1 one at a time, as its GPU path
  runs them (qwen_cuda_cp_step per position).  Its fused two-position variant
  caches its mode per thread on first use (qwen_tts_code_predictor.c:784), so
  a process that runs a quantized code predictor and then a bf16 one takes the
  quantized branch on bf16 weights and crashes.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "qwen3-tts_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
for _k, _v in {"QWEN_NO_BF16DOT": "1", "QWEN_NO_VNNI": "1", "QWEN_NO_SDOT": "1", "QWEN_CP_PREFILL2": "0"}.items():
    os.environ.setdefault(_k, _v)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a engine")
    config.addinivalue_line("markers", "slow: full-size model cases (tens of seconds)")


def gpu_available():
    try:
        import qtts_b200 as Q
        return Q.lib().qtb_device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def have_gpu():
    if not gpu_available():
        pytest.fail("GPU test selected but no CUDA device / engine library is available")
    return True
