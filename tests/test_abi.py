"""CPU checks of the C ABI: the library loads without a GPU, exports every
function include/tla_api.h declares, and its host-side ropeParameters
restatement matches the reference's pinned golden vectors."""
import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "tla_api.h"
ROPE = json.loads((ROOT / "tests" / "golden" / "rope_cases.json").read_text())


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(tla_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(pkg):
    names = declared_functions()
    assert len(names) >= 16
    lib = pkg.lib()
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(pkg.EXPORTS) == names


def test_status_strings_carry_reference_messages(pkg):
    lib = pkg.lib()
    assert lib.tla_status_string(-2).decode() == "RoPE dimension must be a non-negative even integer."
    assert lib.tla_status_string(-7).decode() == "Invalid Llama 3 RoPE frequency range."


@pytest.mark.parametrize("case", ROPE["cases"], ids=[c["name"] for c in ROPE["cases"]])
def test_rope_parameters_match_pinned_transformers(pkg, case):
    from three_llm_b200.attention import rope_parameters

    inv, af = rope_parameters(8, case["theta"], case["scaling"])
    assert np.all(np.abs(inv - np.asarray(case["inv_freq"])) <= 1e-8 + 1e-6 * np.abs(case["inv_freq"]))
    assert af == pytest.approx(case["attention_factor"], abs=5e-7)


def test_rope_parameters_equal_oracle_bitwise(pkg):
    from oracle import oracle
    from three_llm_b200.attention import rope_parameters

    for dim, theta, sc in [(64, 5e5, None), (128, 1e6, None), (64, 1e4, {"type": "linear", "factor": 4}),
                           (128, 5e5, {"type": "llama3", "factor": 8, "original_context_length": 8192,
                                       "low_freq_factor": 1, "high_freq_factor": 4}),
                           (64, 1e4, {"type": "yarn", "factor": 4, "original_context_length": 4096,
                                      "beta_fast": 32, "beta_slow": 1})]:
        a, af = rope_parameters(dim, theta, sc)
        b, bf = oracle.rope_parameters(dim, theta, sc)
        np.testing.assert_array_equal(a, b)
        assert af == bf


def test_rope_rejections_through_abi(pkg):
    from three_llm_b200.attention import rope_parameters

    for args, code in [((3, 1e4, None), "TLA_ERR_ROPE_DIM"), ((8, 1.0, None), "TLA_ERR_ROPE_THETA"),
                       ((8, 1e4, {"type": "linear", "factor": 0.5}), "TLA_ERR_ROPE_FACTOR"),
                       ((8, 1e4, {"type": "llama3", "factor": 4}), "TLA_ERR_LLAMA3_RANGE")]:
        with pytest.raises(pkg.TlaError, match=code):
            rope_parameters(*args)


def test_create_without_device_reports_status(pkg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    assert pkg.lib().tla_create(0, ctypes.byref(h)) == -14  # TLA_ERR_NO_DEVICE
