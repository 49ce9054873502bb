"""Host logic of the Python binding that needs no GPU."""
import numpy as np

import nemoasr_b200 as nb


def test_token_lists_match_row_slices():
    rng = np.random.default_rng(0)
    for B, k in ((1, 0), (1, 5), (7, 0), (256, 3), (256, 60)):
        tok = rng.integers(0, 1025, (B, 128)).astype(np.int32)
        cnt = rng.integers(0, k + 1, B).astype(np.int32)
        got = nb._token_lists(tok, cnt)
        assert got == [tok[i, :cnt[i]].tolist() for i in range(B)]
        assert all(type(t) is int for row in got for t in row)
