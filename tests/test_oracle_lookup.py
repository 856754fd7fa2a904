"""The n-gram drafter oracle (oracle.lookup_ngram) against a literal loop
restatement of engine/lookup11_nw32.cu:17-58 (nested compares, key (l << 20) | i,
max over starts) on small histories, plus known-answer cases."""
import numpy as np
import pytest

import oracle
from thunderllamax_b200.ops import LOOKUP_SCAN_END


def loop_lookup(h, pos, k, e):
    if pos < e:
        return 1000000 + pos, None
    s = [int(h[pos - 8 + j]) for j in range(8)]
    key = 0
    for i in range(0, pos - e + 1):
        l = 0
        while l < 8 and int(h[i + l]) == s[l]:
            l += 1
        if l >= 1:
            key = max(key, (l << 20) | i)
    l = key >> 20
    drafts = None
    if l >= 8:
        i = key & 0xFFFFF
        drafts = np.array([h[i + 8 + j] for j in range(k)], np.int32)
    return l + 1, drafts


def planted_history(rng, n, vocab, plants):
    h = rng.integers(0, vocab, n).astype(np.int32)
    for _ in range(plants):   # copy a random 8..30-token span to a later spot
        ln = int(rng.integers(8, 31))
        if n <= ln:
            break
        a = int(rng.integers(0, n - ln))
        b = int(rng.integers(0, n - ln))
        h[b:b + ln] = h[a:a + ln].copy()
    return h


@pytest.mark.parametrize("k", sorted(LOOKUP_SCAN_END))
def test_oracle_matches_loop_restatement(k):
    e = LOOKUP_SCAN_END[k]
    rng = np.random.default_rng(100 + k)
    for trial in range(40):
        n = int(rng.integers(1, 400))
        h = planted_history(rng, n, int(rng.integers(2, 12)), int(rng.integers(0, 4)))
        # pos at the end, or with the suffix copied from earlier (a sure hit)
        pos = int(rng.integers(0, n + 1))
        if trial % 3 == 0 and n > 40:
            a = int(rng.integers(0, n - 30))
            h[n - 8:n] = h[a:a + 8]
            pos = n
        lh, d = oracle.lookup_ngram(h, pos, k, e)
        lh2, d2 = loop_lookup(h, pos, k, e)
        assert lh == lh2
        assert (d is None and d2 is None) or np.array_equal(d, d2)


def test_known_answers():
    k, e = 10, 19
    # suffix 1..8 occurs at 4 and (later) at 30: the most recent full match wins
    h = np.arange(100, 160, dtype=np.int32)
    h[4:12] = np.arange(1, 9)
    h[30:38] = np.arange(1, 9)
    h[52:60] = np.arange(1, 9)           # the suffix itself (pos = 60)
    lh, d = oracle.lookup_ngram(h, 60, k, e)
    assert lh == 9 and np.array_equal(d, h[38:48])
    # the later copy lies past the scan end (i <= pos - 19 = 41 holds for 30; move it)
    h2 = h.copy()
    h2[30:38] = 0
    h2[40:48] = np.arange(1, 9)           # i = 40 <= 41: still scanned
    lh, d = oracle.lookup_ngram(h2, 60, k, e)
    assert lh == 9 and np.array_equal(d, h2[48:58])
    h2[40:48] = 0
    h2[42:50] = np.arange(1, 9)           # i = 42 > 41: not scanned, i = 4 wins
    lh, d = oracle.lookup_ngram(h2, 60, k, e)
    assert lh == 9 and np.array_equal(d, h2[12:22])
    # partial matches only: l_hist = l + 1, no drafts
    h3 = np.arange(100, 160, dtype=np.int32)
    h3[52:60] = np.arange(1, 9)
    h3[10:15] = np.arange(1, 6)
    assert oracle.lookup_ngram(h3, 60, k, e) == (6, None)
    # nothing matches the first suffix token
    assert oracle.lookup_ngram(np.arange(60, dtype=np.int32), 60, k, e) == (1, None)
    # suffix / scan range undefined
    assert oracle.lookup_ngram(h, 18, k, e) == (1000018, None)
