"""The oracle reproduces the committed golden fixtures bit for bit (CPU).

The fixtures were written by tests/golden/make_golden.py from this oracle;
the reference itself publishes none (no tests in the reference repository).
"""
import numpy as np
import pytest

from harness import (ATTN_FIXTURES, GDN_FIXTURES, load_attn_fixture, load_gdn_fixture,
                     oracle_attention, oracle_gdn)


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_attention_fixture(name):
    inp, out = load_attn_fixture(name)
    assert np.array_equal(oracle_attention(inp), out)


@pytest.mark.parametrize("name", GDN_FIXTURES)
def test_gdn_fixture(name):
    inp, out, state = load_gdn_fixture(name)
    o, s = oracle_gdn(inp)
    assert np.array_equal(o.view(np.uint32), out.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), state.view(np.uint32))
