"""bench.py's --attn workload spec (CPU only)."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_attn_spec_causal_word_and_flag():
    assert bench.parse_attn_spec("1,32,8192,8192,128,causal") == (1, 32, 8192, 8192, 128, True)
    assert bench.parse_attn_spec("4,16,2048,2048,128") == (4, 16, 2048, 2048, 128, False)
    assert bench.parse_attn_spec("4, 16, 2048, 2048, 64, 1")[-1] is True
    assert bench.parse_attn_spec("4,16,2048,2048,64,0")[-1] is False


def test_attn_spec_rejects_bad_field_counts():
    with pytest.raises(ValueError):
        bench.parse_attn_spec("4,16,2048")
    with pytest.raises(ValueError):
        bench.parse_attn_spec("1,2,3,4,5,causal,extra")
