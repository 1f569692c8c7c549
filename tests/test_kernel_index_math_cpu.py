"""CPU restatements of index arithmetic in two kernels, checked exhaustively on small and
ragged sizes: the peer-pull all-gather's thread -> (peer, vector) mapping
(csrc/symmetric.cu: symm_all_gather_kernel) and the MN-major GEMM producer's box count and
expected transaction bytes at the M / N tails (csrc/gemm.cu: gemm_bf16_kernel, LAYOUT != 0)."""
import itertools


def _gather_targets(P, rank, units):
    """(peer, unit) pairs written by the grid-stride loop of symm_all_gather_kernel."""
    others = P - 1
    out = []
    for i in range(others * units):
        w = i // others
        j = i - w * others
        q = j + (1 if j >= rank else 0)
        out.append((q, w))
    return out


def test_all_gather_covers_every_peer_unit_once():
    for P in range(2, 9):
        for rank in range(P):
            for units in (1, 3, 17):
                got = _gather_targets(P, rank, units)
                want = [(q, w) for q in range(P) if q != rank for w in range(units)]
                assert sorted(got) == sorted(want) and len(set(got)) == len(got)
                # consecutive threads read different peers
                assert all(a[0] != b[0] for a, b in zip(got, got[1:]) if P > 2)


BM, BN, BK = 128, 256, 64
A_BYTES, B_BYTES = BM * BK * 2, BN * BK * 2


def _mn_boxes(M, N, mb, nb, layout):
    na = min(BM // 64, (M - mb * BM + 63) // 64) if layout & 1 else 1
    nbx = min(BN // 64, (N - nb * BN + 63) // 64) if layout & 2 else 1
    nbytes = (na * (A_BYTES // 2) if layout & 1 else A_BYTES) + \
             (nbx * (B_BYTES // 4) if layout & 2 else B_BYTES)
    return na, nbx, nbytes


def test_mn_major_boxes_cover_the_tile_and_skip_only_past_the_edge():
    for M, N, layout in itertools.product((40, 128, 136, 200, 8192), (40, 200, 256, 328, 5376), (1, 2, 3)):
        num_m, num_n = -(-M // BM), -(-N // BN)
        for mb in range(num_m):
            for nb in range(num_n):
                na, nbx, nbytes = _mn_boxes(M, N, mb, nb, layout)
                if layout & 1:
                    starts = [mb * BM + 64 * i for i in range(na)]
                    assert all(x < M for x in starts)                 # every box starts inside
                    assert mb * BM + 64 * na >= min(M, (mb + 1) * BM)  # and they cover the rows
                    assert all((x * 2) % 16 == 0 for x in starts)     # TMA x alignment
                if layout & 2:
                    starts = [nb * BN + 64 * i for i in range(nbx)]
                    assert all(x < N for x in starts)
                    assert nb * BN + 64 * nbx >= min(N, (nb + 1) * BN)
                    assert all((x * 2) % 16 == 0 for x in starts)
                assert 0 < nbytes <= A_BYTES + B_BYTES
