"""The reviewed-upstream-source gate: the fingerprint function and the reviewed tables against what the reference's
own ``step_cache.fingerprint_source`` and tables produce (``tests/golden/sources.json``, written by make_golden.py)."""
import functools
import json
from pathlib import Path

from h3b import sources

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "sources.json").read_text())


def test_fingerprint_source_equals_the_reference():
    for text, want in zip(GOLDEN["samples"], GOLDEN["fingerprints"]):
        assert sources.fingerprint_source(text) == want, text


def test_reviewed_tables_equal_the_reference():
    assert sources.REVIEWED == GOLDEN["consumer_expected"]
    assert {k: list(v) for k, v in sources.CONSUMER_SITE_SOURCES.items()} == GOLDEN["consumer_sites"]
    assert sources.REVIEWED_EXTRA == GOLDEN["quant_expected_extra"]
    assert {k: list(v) for k, v in sources.QUANT_SITE_SOURCES.items()} == GOLDEN["quant_sites"]
    assert sources.OUTQ_REVIEWED == GOLDEN["outq_expected"]


def _upstream(x):
    # a comment the fingerprint ignores
    return x + 1


def test_fingerprint_follows_wraps_and_ignores_comments():
    @functools.wraps(_upstream)
    def wrapper(*a):
        return _upstream(*a)

    def rewrapped(x):
        return x + 1

    assert sources.fingerprint(wrapper) == sources.fingerprint(_upstream)
    assert sources.fingerprint(rewrapped) != sources.fingerprint(_upstream)     # the def line differs
    assert sources.fingerprint(len) is None                                      # no Python source
    assert sources.changed(("a", "b"), {"a": "1", "b": "3"}, {"a": "1", "b": "2"}) == ["b 3 (reviewed 2)"]
