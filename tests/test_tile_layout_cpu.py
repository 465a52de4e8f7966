"""Index arithmetic of the edge-row GEMM path (pymolecular_b200/csrc/edge_rows.cu),
restated on the host: the tile-major operand layout, the per-warp store staging
(`store_rows64`) and the coalesced side-row loads (`load_rows128`).

Each restatement mirrors one formula of the kernels; the checks are the
properties the kernels rely on: every 16-byte chunk of a destination is written
exactly once by the lane that owns it, each global instruction covers whole row
pieces, and no 8-lane group of a shared-memory access hits one 16-byte bank group
twice.
"""
import itertools


def sw128_chunk(row, col):
    """Byte offset of the 16-byte chunk holding bf16 column `col` of row `row`
    inside one 128-row x 64-column block of a tile (the 128-byte swizzle)."""
    return row * 128 + (((col % 64) // 8) ^ (row % 8)) * 16


def tile_piece_chunk(el, cs, p, c):
    """st_tile_piece: logical chunk c (features 64 cs + 32 p + 8 c ..) of row el
    goes to the 64-byte group at ((4 p) ^ (el & 4)) * 16 of the row, position c ^ (el & 3)."""
    group = (((p << 2) ^ (el & 4)) << 4)
    return cs * 128 * 128 + el * 128 + group + ((c ^ (el & 3)) << 4)


def test_tile_piece_matches_the_swizzled_block_layout():
    for el, cs, p, c in itertools.product(range(128), range(4), range(2), range(4)):
        col = 64 * cs + 32 * p + 8 * c
        assert tile_piece_chunk(el, cs, p, c) == cs * 128 * 128 + sw128_chunk(el, col)


def test_tile_pieces_cover_each_block_once():
    seen = set()
    for el, cs, p, c in itertools.product(range(128), range(4), range(2), range(4)):
        off = tile_piece_chunk(el, cs, p, c)
        assert off not in seen
        seen.add(off)
    assert seen == {16 * k for k in range(4 * 128 * 128 // 16)}


def _bank_group(addr):
    return (addr // 16) % 8


def test_store_staging_is_a_conflict_free_bijection():
    """store_rows64: lane l writes its row's chunk c at l*64 + ((c ^ ((l >> 1) & 3)) << 4)
    and lane l reads back chunk (l & 3) of row 8 k + (l >> 2)."""
    def wslot(lane, c):
        return lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)
    slots = {wslot(l, c): (l, c) for l in range(32) for c in range(4)}
    assert len(slots) == 128 and max(slots) < 2048
    for c in range(4):   # writes: each 8-lane group hits 8 distinct bank groups
        for g in range(4):
            assert len({_bank_group(wslot(l, c)) for l in range(8 * g, 8 * g + 8)}) == 8
    got = set()
    for k in range(4):
        reads = []
        for lane in range(32):
            hr, cc = 8 * k + (lane >> 2), lane & 3
            addr = hr * 64 + ((cc ^ ((hr >> 1) & 3)) << 4)
            assert slots[addr] == (hr, cc)          # the chunk written by row hr's lane
            reads.append(addr)
            got.add((hr, cc))
        for g in range(4):
            assert len({_bank_group(a) for a in reads[8 * g:8 * g + 8]}) == 8
        # one global instruction: rows 8k .. 8k+7, four lanes (64 bytes) each
        rows = [8 * k + (lane >> 2) for lane in range(32)]
        assert sorted(set(rows)) == list(range(8 * k, 8 * k + 8))
    assert len(got) == 128


def test_side_row_loads_hand_every_lane_its_own_row():
    """load_rows128: in round h, lane l loads chunk (l & 7) of row 16 h + 4 k + (l >> 3)
    into slot rr * 128 + ((c ^ (rr & 7)) << 4); lanes 16 h .. 16 h + 15 read back
    their own row's eight chunks."""
    for h in range(2):
        stg = {}
        for k in range(4):
            addrs = []
            for lane in range(32):
                rr, c = 4 * k + (lane >> 3), lane & 7
                a = rr * 128 + ((c ^ (rr & 7)) << 4)
                assert a not in stg
                stg[a] = (16 * h + rr, c)
                addrs.append(a)
            for g in range(4):
                assert len({_bank_group(a) for a in addrs[8 * g:8 * g + 8]}) == 8
        assert len(stg) == 128 and max(stg) < 2048
        for lane in range(16 * h, 16 * h + 16):
            rr = lane & 15
            for c in range(8):
                assert stg[rr * 128 + ((c ^ (rr & 7)) << 4)] == (lane, c)
        # reads: 16 lanes per chunk index, at most two per bank group
        for c in range(8):
            groups = [_bank_group(rr * 128 + ((c ^ (rr & 7)) << 4)) for rr in range(16)]
            assert max(groups.count(b) for b in set(groups)) <= 2


def test_weight_gradient_slabs_tile_the_operand_blocks():
    """rows_wgrad_kernel: slab q of a tile copies, from each 16 KB column block b,
    the 4 KB row range q * 4096 .. + 4095 (rows 32 q .. 32 q + 31); the four slabs
    of a tile cover the tile once and keep row % 8 (the swizzle phase)."""
    covered = set()
    for q, b in itertools.product(range(4), range(4)):
        start = b * 16384 + q * 4096
        for off in range(start, start + 4096, 128):
            row = (off - b * 16384) // 128
            assert row // 32 == q and (off - start) // 128 % 8 == row % 8
            covered.add(off)
    assert covered == set(range(0, 65536, 128))
