"""Host-side work split of the batched matmul (gguf_cuda_matmul_plan): the
(row tile, super-block) units are split evenly over at most one CTA per SM
and about four CTAs per row tile, and the partial-sum slots per tile cover
every CTA that shares the tile.
Runs without a GPU."""
import pytest

import pk_b200


def brute(rows, nsb, sms):
    tiles = (rows + 127) // 128
    U = tiles * nsb
    G = min(U, sms, 4 * tiles)
    owner = []
    for c in range(G):
        owner += [c] * ((c + 1) * U // G - c * U // G)
    assert len(owner) == U
    maxp = max(len(set(owner[T * nsb:(T + 1) * nsb])) for T in range(tiles))
    return G, maxp


@pytest.mark.parametrize("rows,cols", [(1, 256), (128, 256), (130, 4096), (2048, 2048), (4096, 4096),
                                       (11008, 4096), (4096, 11008), (32000, 4096), (128256, 4096), (5, 40960)])
@pytest.mark.parametrize("sms", [1, 7, 148])
def test_plan_matches_even_split(rows, cols, sms):
    assert pk_b200.matmul_plan(rows, cols // 256, sms) == brute(rows, cols // 256, sms)
