"""The attention kernel's work split (cb_attention_schedule, no GPU needed): every
128-query tile of every (batch, head) is in exactly one CTA's list, the lists are
balanced, and each CTA walks its tiles head by head (or chunk of heads by chunk), the
latest query tiles first."""
import ctypes as C

import numpy as np
import pytest

from rustane_b200 import bridge as B


def schedule(batch, heads, kv_heads, seq, sms=148):
    lib = B.load_library()
    grid, n = C.c_int32(), C.c_size_t()
    rc = lib.cb_attention_schedule(batch, heads, kv_heads, seq, sms, None, 0,
                                   C.byref(grid), C.byref(n))
    assert rc == B.CB_ERR_INVALID_ARG and n.value > 0  # size query
    table = (C.c_int32 * n.value)()
    rc = lib.cb_attention_schedule(batch, heads, kv_heads, seq, sms, table, n.value,
                                   C.byref(grid), C.byref(n))
    assert rc == B.CB_OK
    t = np.frombuffer(table, dtype=np.int32).copy()
    g = grid.value
    off, items = t[:g + 1], t[g + 1:]
    return g, [items[off[c]:off[c + 1]] for c in range(g)]


SHAPES = [(64, 12, 12, 512), (8, 12, 12, 512), (1, 12, 12, 512), (8, 32, 32, 512),
          (8, 40, 40, 512), (16, 52, 52, 2048), (2, 6, 3, 2048), (3, 2, 1, 128),
          (1, 1, 1, 128), (4, 8, 2, 384)]


@pytest.mark.parametrize("batch,heads,kv,seq", SHAPES)
def test_every_tile_once_and_balanced(bridge_lib, batch, heads, kv, seq):
    n_qt = seq // 128
    n_items = batch * heads * n_qt
    g, lists = schedule(batch, heads, kv, seq)
    assert g == min(n_items, 2 * 148)
    flat = np.concatenate(lists)
    assert np.array_equal(np.sort(flat), np.arange(n_items))
    cost = [sum(2 * (w % n_qt + 1) + 1 for w in lst) for lst in lists]
    heaviest = 2 * n_qt + 1
    # no CTA ends more than two of the heaviest tiles after the mean
    assert max(cost) <= np.mean(cost) + 2 * heaviest


def _head_major_snake_max(batch, heads, seq, g):
    n_qt = seq // 128
    loads = np.zeros(g)
    for k in range(batch * heads * n_qt):
        rd, c = divmod(k, g)
        loads[g - 1 - c if rd & 1 else c] += 2 * (n_qt - 1 - k % n_qt + 1) + 1
    return loads.max()


@pytest.mark.parametrize("batch,heads,kv,seq", SHAPES)
def test_tiles_run_in_head_order_latest_first(bridge_lib, batch, heads, kv, seq):
    """Each CTA walks its tiles in the order of one of the two splits: head-major (heads
    in order, latest tile first) or chunks of heads whose K and V fit in 8 MB (chunks in
    order, latest tiles of the chunk first); the table never does worse than the
    head-major split by the cost model."""
    n_qt = seq // 128
    hb = batch * heads
    chunk = max(1, min(hb, int(8 * 2**20 / (seq * 128 * 4 / (heads // kv)))))
    g, lists = schedule(batch, heads, kv, seq)
    head_major = all([(w // n_qt, n_qt - 1 - w % n_qt) for w in lst] ==
                     sorted((w // n_qt, n_qt - 1 - w % n_qt) for w in lst) for lst in lists)
    chunked = all([((w // n_qt) // chunk, n_qt - 1 - w % n_qt) for w in lst] ==
                  sorted(((w // n_qt) // chunk, n_qt - 1 - w % n_qt) for w in lst)
                  for lst in lists)
    assert head_major or chunked
    cost = max(sum(2 * (w % n_qt + 1) + 1 for w in lst) for lst in lists)
    assert cost <= _head_major_snake_max(batch, heads, seq, g)


def test_rejects_bad_shapes(bridge_lib):
    lib = B.load_library()
    grid, n = C.c_int32(), C.c_size_t()
    for args in [(0, 12, 12, 512), (1, 12, 5, 512), (1, 12, 12, 500), (1, 12, 12, 64)]:
        assert lib.cb_attention_schedule(*args, 148, None, 0, C.byref(grid),
                                         C.byref(n)) == B.CB_ERR_INVALID_ARG
