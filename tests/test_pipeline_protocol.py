"""Models of the kernels' ring protocols, checked on the CPU (no kernel runs here).

The kernels in foreswe_gpu_optimization_b200/csrc/geoattn_kernels.cuh hand buffers between their TMA, MMA and
element-wise warps through mbarrier rings. Some of those hand-overs are easy to get wrong and fail on the GPU only as
a bounded-wait timeout or as results that differ between runs, so their arithmetic is restated here:

* pooled fp32 kernels (head dim 64): the landing of a tile's tensor-memory operand takes every slot of a chunk ring
  once, completing an `empty` phase per slot but no `full` phase; the consumer's `full` parity skips the landings;
* the forward's pass B with chunk pairs: V of chunk c is loaded after the K of chunk c + VLAG. With wide head dims a
  pair takes NDC ring slots, more than the ring holds, and a lag of NSB - 1 deadlocks (seen on the GPU as expired
  bounded waits); the kernels use NSB - PAIR there;
* the wide row pass's sweep 2 with chunk pairs: the transposed K chunks for dQ trail the slots by one pair;
* the wide key pass with query-chunk pairs: a chunk's records load before the next pair's slots;
* the BF16 key pass's dS^T scratch stores trail the query-chunk loads by at most NQ + NST - 1 chunks;
* the BF16 forward over several tiles: pass B's V loads may lag the K loads by 1 ... NSB + NK - 1 chunks (the kernel
  uses NSB - 1); with Q in tensor memory and K in a ring of chunk pairs (head dims up to 128) by 0 ... NSB + 2 NK - 2;
* the forwards with a single score pass (bf16, and fp32 at head dim 64 with its Q landing in the K ring);
* the wide key pass's dS^T stores (fp32 above head dim 64), trailing the loads by one chunk.
"""
import pytest

NSB = 4     # forward score buffers in tensor memory
PAIR = 2    # 32-key chunks per score MMA (pooled and wide fp32 forward)


def _ring_positions(n_tiles, n_chunks, depth, land):
    """Yield (tile, position, is_landing) in the producer's order: `land` landing positions, then the chunks."""
    pos = 0
    for it in range(n_tiles):
        for _ in range(land):
            yield it, pos, True
            pos += 1
        for _ in range(n_chunks):
            yield it, pos, False
            pos += 1


@pytest.mark.parametrize("depth,chunks_per_tile", [(2, 11), (2, 1), (2, 2), (3, 16), (4, 22), (4, 2), (3, 8)])
def test_pooled_ring_parities(depth, chunks_per_tile):
    """Every wait of the pooled rings targets exactly the phase it needs: `empty` waits (TMA) the release of the
    previous use of the slot, `full` waits (MMA) the k-th chunk load of the slot, k = pos / depth - (tile + 1)."""
    released = [0] * depth   # empty phases completed per slot (landings and chunks)
    loads = [0] * depth      # full phases completed per slot (chunk loads only)
    for it, pos, landing in _ring_positions(5, chunks_per_tile, depth, depth):
        slot = pos % depth
        # the producer waits for phase pos / depth - 1 of empty[slot]: the previous use of the slot is released
        assert released[slot] == pos // depth
        if not landing:
            k = loads[slot]
            loads[slot] += 1
            # the consumer's parity formula for full[slot]
            assert (pos // depth - (it + 1)) == k
        released[slot] += 1


def _forward_order(nch, ndc, nk, vlag):
    """Pass A and pass B of one forward tile as three cooperating programs; returns None or the deadlock state.

    TMA: K slot loads for each chunk pair (ndc head-dim slots per pair through an nk-slot ring); in pass B, after the
    pair holding chunk cc, V of chunk cc - vlag (two V buffers). MMA: score MMAs per pair (both score buffers free),
    keeping pass B's scores up to NSB - 1 chunks ahead, then P.V of chunk c (needs P staged and V loaded).
    Element-wise: releases score buffers; stages P of chunk c once P.V of c - 2 ran."""
    st = dict(kload=0, kcons=0, vload=0, pv=0, s_issued=0, s_released=0, p_staged=0)

    def tma():
        for pass_ in range(2):
            for c in range(0, nch, PAIR):
                for _ in range(ndc):
                    yield lambda: st["kload"] - st["kcons"] < nk
                    st["kload"] += 1
                if pass_ == 1:
                    for cc in range(c, c + PAIR):
                        if cc >= vlag:
                            v = cc - vlag
                            yield lambda v=v: st["pv"] >= v - 1
                            st["vload"] = v + 1
            if pass_ == 1:
                for v in range(max(0, nch - vlag), nch):
                    yield lambda v=v: st["pv"] >= v - 1
                    st["vload"] = v + 1

    def mma():
        sc = 0

        def issue():
            nonlocal sc
            yield lambda: st["s_released"] >= sc + PAIR - NSB
            for _ in range(ndc):
                yield lambda: st["kload"] > st["kcons"]
                st["kcons"] += 1
            sc += PAIR
            st["s_issued"] = sc

        for _ in range(0, nch, PAIR):
            yield from issue()
        nb = 0
        for c in range(nch):
            while nb < nch and nb + PAIR - 1 < c + NSB:
                yield from issue()
                nb += PAIR
            yield lambda c=c: st["p_staged"] > c and st["vload"] > c
            st["pv"] = c + 1

    def ew():
        for c in range(0, nch, PAIR):
            yield lambda c=c: st["s_issued"] >= c + PAIR
            st["s_released"] = c + PAIR
        for c in range(nch):
            yield lambda c=c: st["s_issued"] >= nch + c + 1
            st["s_released"] = nch + c + 1
            yield lambda c=c: st["pv"] >= c - 1
            st["p_staged"] = c + 1

    progs = [tma(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * 3
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


# (head-dim slots per pair, K ring slots): pooled D = 64, wide D = 128, wide D = 192
CONFIGS = [(1, 3, NSB - 1), (4, 3, NSB - PAIR), (6, 2, NSB - PAIR)]


@pytest.mark.parametrize("ndc,nk,vlag", CONFIGS, ids=["pooled-d64", "wide-d128", "wide-d192"])
@pytest.mark.parametrize("nch", [2, 4, 6, 10, 16, 48])
def test_forward_pair_order_has_no_deadlock(ndc, nk, vlag, nch):
    assert _forward_order(nch, ndc, nk, vlag) is None


@pytest.mark.parametrize("ndc,nk", [(4, 3), (6, 2)], ids=["wide-d128", "wide-d192"])
def test_forward_wide_pairs_deadlock_with_the_unpaired_lag(ndc, nk):
    """The lag of the unpaired kernels (NSB - 1) stalls the wide pair schedule: the planted mistake is caught."""
    assert _forward_order(16, ndc, nk, NSB - 1) is not None


def _key_pass_wide_order(n, ndc, nrs, records_first, slag=None):
    """Wide fp32 key pass, one tile, query chunks in pairs: per chunk the TMA loads its row records (two buffers),
    before chunk 0 and each odd chunk the slots of the next pair (2*ndc head-dim slots through an nrs-slot ring), then
    the chunk's transposed Q/dO (one buffer, free once the previous chunk's dV/dK ran). The MMA issues a pair into both
    score buffers, the next pair after the first chunk's dV/dK. The element-wise warps need a chunk's scores and its
    records before they free its score buffer, and stage P2^T/dS^T (one buffer). With `slag` (the dS-scratch backward)
    the TMA also stores the staged dS^T tile of chunk c - slag after chunk c's transposed Q/dO, and the staging buffer
    is free for the next chunk only once both its dV/dK MMAs and its store have read it. Returns None or the deadlock
    state."""
    st = dict(sl=0, sc=0, s_iss=0, s_rel=0, staged=0, dvdk=0, qt=0, rec=0, rec_read=0, stored=0)

    def tma():
        def slots():
            for _ in range(2 * ndc):
                yield lambda: st["sl"] - st["sc"] < nrs
                st["sl"] += 1

        for c in range(n):
            def records(c=c):
                yield lambda: st["rec_read"] >= c - 1
                st["rec"] = c + 1

            if records_first:
                yield from records()
            first = 0 if c == 0 else (c + 1 if c % 2 else -1)
            if 0 <= first < n:
                yield from slots()
            yield lambda c=c: st["dvdk"] >= c
            st["qt"] = c + 1
            if not records_first:
                yield from records()
            if slag is not None and c >= slag:
                yield lambda g=c - slag: st["staged"] > g
                st["stored"] = c - slag + 1
        if slag is not None:
            for g in range(max(0, n - slag), n):
                yield lambda g=g: st["staged"] > g
                st["stored"] = g + 1

    def mma():
        def issue(j):
            yield lambda: st["s_rel"] >= 2 * j
            for _ in range(2 * ndc):
                yield lambda: st["sl"] > st["sc"]
                st["sc"] += 1
            st["s_iss"] = 2 * j + 2

        yield from issue(0)
        for c in range(n):
            yield lambda c=c: st["staged"] > c and st["qt"] > c
            st["dvdk"] = c + 1
            if c % 2 == 0 and c + 2 < n:
                yield from issue(c // 2 + 1)

    def ew():
        for c in range(n):
            yield lambda c=c: st["s_iss"] > c and st["rec"] > c
            st["s_rel"] = c + 1
            st["rec_read"] = c + 1
            yield lambda c=c: st["dvdk"] >= c and (slag is None or st["stored"] >= c)
            st["staged"] = c + 1

    progs = [tma(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * 3
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


@pytest.mark.parametrize("ndc", [4, 6], ids=["d128", "d192"])
@pytest.mark.parametrize("n", [2, 4, 10, 48])
def test_key_pass_wide_order(ndc, n):
    """Records before the slots (the kernels' order); loaded after the transposed Q/dO instead, the element-wise warps
    cannot free the odd chunk's scores while the TMA waits for the next pair's slots to drain, and the pipeline stops
    as soon as a tile has two pairs (it did on the GPU; the planted order is caught)."""
    assert _key_pass_wide_order(n, ndc, 3, records_first=True) is None
    if n >= 4:
        assert _key_pass_wide_order(n, ndc, 3, records_first=False) is not None


@pytest.mark.parametrize("ndc", [4, 6], ids=["d128", "d192"])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 10, 48])
def test_key_pass_wide_store_lag(ndc, n):
    """ColsCfg<false, DP > 64, true>: one query-chunk buffer and one staging buffer (NQ = NST = 1), the dS^T stores
    trailing by one chunk (SLAG = 1 = NQ + NST - 1); a store two chunks behind waits on a staging that waits on it."""
    assert _key_pass_wide_order(n, ndc, 3, records_first=True, slag=1) is None
    if n >= 3:
        assert _key_pass_wide_order(n, ndc, 3, records_first=True, slag=2) is not None


def _rows_wide_pair_order(nch, ndc, nkv, kt_lag_pairs, nds=1):
    """Wide fp32 row pass, one tile: two sweeps of chunk-pair S/dP MMAs (2*ndc head-dim slots per pair through an
    nkv-slot ring, four score buffers); sweep 2 issues the next pair's scores before this pair's dQ MMAs, which need
    the staged dS and the transposed K chunk (nds buffers, each free once the previous use's dQ ran). The TMA loads
    the K^T chunks of a pair `kt_lag_pairs` pairs after its slots. Returns None or the deadlock state."""
    st = dict(kload=0, kcons=0, s_iss=0, s_rel=0, staged=0, dq=0, kt=0)

    def tma():
        for sweep in range(2):
            for c in range(0, nch, PAIR):
                for _ in range(2 * ndc):
                    yield lambda: st["kload"] - st["kcons"] < nkv
                    st["kload"] += 1
                if sweep == 1 and c >= PAIR * kt_lag_pairs:
                    for cc in range(c - PAIR * kt_lag_pairs, c - PAIR * kt_lag_pairs + PAIR):
                        yield lambda cc=cc: st["dq"] >= cc - nds + 1
                        st["kt"] = cc + 1
            if sweep == 1:
                for cc in range(max(0, nch - PAIR * kt_lag_pairs), nch):
                    yield lambda cc=cc: st["dq"] >= cc - nds + 1
                    st["kt"] = cc + 1

    def mma():
        sc = 0

        def issue():
            nonlocal sc
            yield lambda: st["s_rel"] >= sc + PAIR - NSB
            for _ in range(2 * ndc):
                yield lambda: st["kload"] > st["kcons"]
                st["kcons"] += 1
            sc += PAIR
            st["s_iss"] = sc

        for _ in range(0, nch, PAIR):
            yield from issue()
        yield from issue()
        for c in range(0, nch, PAIR):
            if c + PAIR < nch:
                yield from issue()
            for cc in range(c, c + PAIR):
                yield lambda cc=cc: st["staged"] > cc and st["kt"] > cc
                st["dq"] = cc + 1

    def ew():
        for c in range(nch):
            yield lambda c=c: st["s_iss"] > c
            st["s_rel"] = c + 1
        for c in range(nch):
            yield lambda c=c: st["s_iss"] > nch + c
            st["s_rel"] = nch + c + 1
            yield lambda c=c: st["dq"] >= c - nds + 1
            st["staged"] = c + 1

    progs = [tma(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * 3
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


@pytest.mark.parametrize("ndc", [4, 6], ids=["d128", "d192"])
@pytest.mark.parametrize("nch", [2, 4, 6, 16, 48])
def test_rows_wide_pair_order(ndc, nch):
    """The K^T loads trail the slots by one pair (the kernels' order); loaded with their own pair, a dQ MMA that must
    follow the next pair's scores holds the single K^T buffer and the pipeline stops (the planted order is caught)."""
    assert _rows_wide_pair_order(nch, ndc, 3, kt_lag_pairs=1) is None
    if nch >= 4:
        assert _rows_wide_pair_order(nch, ndc, 3, kt_lag_pairs=0) is not None


def _key_pass_bf16_order(nch, n_tiles, nq, nsb, nst, npr, slag, nr=2):
    """The BF16 key pass with the dS^T scratch stores (geoattn_bwd_cols_kernel<true, DP, true>) over several tiles of
    one CTA, as four cooperating programs; returns None or the deadlock state.

    TMA: per tile the K/V blocks (once the previous tile's last S^T/dP^T MMAs were issued), then per chunk the Q/dO
    tile (nq-slot ring, released by the chunk's dV/dK MMAs), its row records (nr-slot ring, released by the
    element-wise warps) and the store of chunk c - slag's staged dS^T tile (after the element-wise warps staged it;
    the store is the tile's second release). Prior loader: nprior-slot ring of prior tiles. MMA: S^T/dP^T of a chunk
    (its Q/dO loaded, a score buffer free), up to nsb chunks ahead; dV/dK of a chunk (its tiles staged), which
    releases its Q/dO slot and the staging tile; `done` after the tile's last dV/dK. Element-wise warps: per chunk
    wait scores, prior and records, release them, wait for the staging tile (both releases of chunk - nst), stage;
    at the tile's end wait for `done` and for the last staged tiles' stores."""
    st = dict(kv_loaded=0, kv_released=0, q_loaded=0, q_released=0, rec_loaded=0, rec_released=0, pr_loaded=0,
              pr_released=0, s_issued=0, s_released=0, t_staged=0, t_mma=0, t_store=0, done=0)

    def tma():
        for it in range(n_tiles):
            yield lambda it=it: st["kv_released"] >= it
            st["kv_loaded"] = it + 1
            g0 = it * nch
            for c in range(nch):
                gc = g0 + c
                yield lambda gc=gc: st["q_released"] >= gc + 1 - nq
                st["q_loaded"] = gc + 1
                yield lambda gc=gc: st["rec_released"] >= gc + 1 - nr
                st["rec_loaded"] = gc + 1
                if c >= slag:
                    yield lambda g=gc - slag: st["t_staged"] >= g + 1
                    st["t_store"] = gc - slag + 1
            for c in range(max(0, nch - slag), nch):
                yield lambda g=g0 + c: st["t_staged"] >= g + 1
                st["t_store"] = g0 + c + 1

    def prior():
        for gc in range(n_tiles * nch):
            yield lambda gc=gc: st["pr_released"] >= gc + 1 - npr
            st["pr_loaded"] = gc + 1

    def mma():
        def issue(gc):
            yield lambda: st["q_loaded"] >= gc + 1 and st["s_released"] >= gc + 1 - nsb
            st["s_issued"] = gc + 1

        for it in range(n_tiles):
            g0 = it * nch
            yield lambda it=it: st["kv_loaded"] >= it + 1
            yield from issue(g0)
            if nch == 1:
                st["kv_released"] = it + 1
            for c in range(nch):
                gc = g0 + c
                if nsb == 2 and c + 1 < nch:
                    yield from issue(gc + 1)
                    if c + 2 == nch:
                        st["kv_released"] = it + 1
                yield lambda gc=gc: st["t_staged"] >= gc + 1
                st["t_mma"] = gc + 1
                st["q_released"] = gc + 1
                if nsb == 1 and c + 1 < nch:
                    yield from issue(gc + 1)
                    if c + 2 == nch:
                        st["kv_released"] = it + 1
            st["done"] = it + 1

    def ew():
        for it in range(n_tiles):
            g0 = it * nch
            for c in range(nch):
                gc = g0 + c
                yield lambda gc=gc: (st["s_issued"] >= gc + 1 and st["pr_loaded"] >= gc + 1
                                     and st["rec_loaded"] >= gc + 1)
                st["s_released"] = st["rec_released"] = st["pr_released"] = gc + 1
                yield lambda gc=gc: st["t_mma"] >= gc + 1 - nst and st["t_store"] >= gc + 1 - nst
                st["t_staged"] = gc + 1
            last = g0 + nch
            yield lambda it=it, last=last: st["done"] >= it + 1 and st["t_mma"] >= last and st["t_store"] >= last

    progs = [tma(), prior(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * len(progs)
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


# ColsCfg<true, DP> ring depths: (NQ, NSB, NST, NPR); the stores trail by SLAG = NQ - 1 (1 when NQ = 1)
BF16_COLS = {64: (3, 2, 2, 2), 128: (3, 2, 1, 1), 192: (1, 1, 1, 1)}


@pytest.mark.parametrize("D", [64, 128, 192])
@pytest.mark.parametrize("nch", [1, 2, 3, 8])
def test_key_pass_bf16_store_lag_has_no_deadlock(D, nch):
    nq, nsb, nst, npr = BF16_COLS[D]
    slag = nq - 1 if nq > 1 else 1
    assert _key_pass_bf16_order(nch, 4, nq, nsb, nst, npr, slag) is None


@pytest.mark.parametrize("D", [64, 128, 192])
def test_key_pass_bf16_store_lag_bound(D):
    """The load of chunk c waits (through the dV/dK MMAs and the staging of chunk c - NQ) for the store of chunk
    c - NQ - NST: a lag up to NQ + NST - 1 runs, one more stops the pipeline (the planted mistake is caught)."""
    nq, nsb, nst, npr = BF16_COLS[D]
    bound = nq + nst - 1
    assert all(_key_pass_bf16_order(n, 4, nq, nsb, nst, npr, bound) is None for n in (1, 2, 3, 5, 8, 16))
    assert _key_pass_bf16_order(16, 4, nq, nsb, nst, npr, bound + 1) is not None


def _forward_bf16_order(nch, n_tiles, nk, npr, vlag, nsb=NSB):
    """The BF16 forward (geoattn_fwd_kernel<true, DP>) over several tiles of one CTA as four cooperating programs;
    returns None or the deadlock state.

    TMA: per tile the Q block (once the previous tile's last score MMA was issued), then K of every chunk through an
    nk-slot ring in pass A and again in pass B, where V of chunk c - vlag follows K of chunk c (two V buffers, each
    freed by its P.V MMA). Prior loader: pass B's prior tiles through an npr-slot ring. MMA: pass A's score MMAs
    (K loaded, a score buffer free), then pass B keeping its scores up to nsb chunks ahead of the P.V MMAs (Q is
    released after the tile's last score MMA), P.V of chunk c once P(c) is staged and V(c) loaded, `ofull` after the
    last. Element-wise warps: pass A frees the score buffers (two chunks at a time); pass B per chunk waits scores and
    prior, frees them, waits for the P buffer (P.V of c - 2 done), stages P; then waits `ofull`."""
    st = dict(q_loaded=0, q_released=0, k_loaded=0, k_used=0, v_loaded=0, pv=0, pr_loaded=0, pr_released=0,
              s_issued=0, s_released=0, p_staged=0, ofull=0)

    def tma():
        for it in range(n_tiles):
            yield lambda it=it: st["q_released"] >= it
            st["q_loaded"] = it + 1
            vbase = it * nch

            def load_v(cv):
                yield lambda: st["pv"] >= vbase + cv - 1        # V buffer of chunk cv - 2 free
                st["v_loaded"] = vbase + cv + 1

            for pass_ in range(2):
                for c in range(nch):
                    yield lambda: st["k_used"] >= st["k_loaded"] + 1 - nk
                    st["k_loaded"] += 1
                    if pass_ == 1 and c >= vlag:
                        yield from load_v(c - vlag)
                if pass_ == 1:
                    for cv in range(max(0, nch - vlag), nch):
                        yield from load_v(cv)

    def prior():
        for g in range(n_tiles * nch):
            yield lambda g=g: st["pr_released"] >= g + 1 - npr
            st["pr_loaded"] = g + 1

    def mma():
        def issue():
            yield lambda: (st["k_loaded"] >= st["k_used"] + 1 and st["s_released"] >= st["s_issued"] + 1 - nsb)
            st["k_used"] += 1
            st["s_issued"] += 1

        for it in range(n_tiles):
            yield lambda it=it: st["q_loaded"] >= it + 1
            for _ in range(nch):
                yield from issue()
            nb = 0
            for c in range(nch):
                while nb < nch and nb < c + nsb:
                    yield from issue()
                    nb += 1
                    if nb == nch:
                        st["q_released"] = it + 1
                g = it * nch + c
                yield lambda g=g: st["p_staged"] >= g + 1 and st["v_loaded"] >= g + 1
                st["pv"] = g + 1
            st["ofull"] = it + 1

    def ew():
        s = 0
        for it in range(n_tiles):
            for c in range(0, nch, 2):
                two = 2 if c + 1 < nch else 1
                yield lambda s=s, two=two: st["s_issued"] >= s + two
                s += two
                st["s_released"] = s
            for c in range(nch):
                g = it * nch + c
                yield lambda s=s, g=g: st["s_issued"] >= s + 1 and st["pr_loaded"] >= g + 1
                s += 1
                st["s_released"] = s
                st["pr_released"] = g + 1
                yield lambda g=g: st["pv"] >= g - 1
                st["p_staged"] = g + 1
            yield lambda it=it: st["ofull"] >= it + 1

    progs = [tma(), prior(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * len(progs)
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


# FwdCfg<true, DP>: (NK, NPR); V loads lag the K loads by NSB - 1 chunks
BF16_FWD = {64: (3, 2), 128: (3, 2), 192: (2, 1)}


@pytest.mark.parametrize("D", [64, 128, 192])
@pytest.mark.parametrize("nch", [1, 2, 3, 4, 5, 8])
def test_forward_bf16_order_has_no_deadlock(D, nch):
    nk, npr = BF16_FWD[D]
    assert _forward_bf16_order(nch, 3, nk, npr, NSB - 1) is None


@pytest.mark.parametrize("D", [64, 128, 192])
def test_forward_bf16_v_lag_range(D):
    """In pass B the TMA warp loads K(x) and then V(x - VLAG); V(y) waits for P.V(y - 2) (two V buffers), and P.V(c)
    comes after the score MMAs up to chunk c + NSB - 1. Lower bound: K(c + NSB - 1) follows V(c + NSB - 2 - VLAG),
    which waits for P.V(c + NSB - 4 - VLAG), so VLAG >= NSB - 3 = 1. Upper bound: V(c) follows K(c + VLAG), which needs
    the ring slot of K(c + VLAG - NK), free once that chunk's score MMA is issued, so VLAG <= NSB + NK - 1. Lags in
    that range run; 0 and NSB + NK stop (the planted mistakes are caught)."""
    nk, npr = BF16_FWD[D]
    sizes = (1, 2, 3, 4, 5, 8, 16)
    for vlag in range(1, NSB + nk):
        assert all(_forward_bf16_order(n, 3, nk, npr, vlag) is None for n in sizes), vlag
    assert _forward_bf16_order(16, 3, nk, npr, 0) is not None
    assert _forward_bf16_order(16, 3, nk, npr, NSB + nk) is not None


def _forward_pooled_bf16_order(nch, n_tiles, nk, npr, vlag, nsb=NSB):
    """The pooled BF16 forward (geoattn_fwd_kernel<true, DP <= 128>) over several tiles as four cooperating programs;
    returns None or the deadlock state.

    Q lands in the shared-memory pool that otherwise holds the ring of K chunk pairs (nk pair slots): the landing
    takes the ring's next nk positions (each waits for the release of its previous use), the MMA warp copies Q into
    tensor memory, drains the copies through the next score buffer (which must be free) and releases the nk
    positions. Each score MMA covers a pair of chunks into two adjacent score buffers (both free) and releases its K
    pair's ring position. Pass B loads V of chunk cc - vlag after the K pair holding cc (two V buffers, each freed by
    its P.V MMA); the MMA warp keeps pass B's scores up to nsb chunks ahead of the P.V MMAs. Prior loader and
    element-wise warps as in the unpooled model."""
    st = dict(pos=0, released=0, q_loaded=0, pairs_loaded=0, pairs_used=0, v_loaded=0, pv=0, pr_loaded=0,
              pr_released=0, s_issued=0, s_released=0, p_staged=0, ofull=0)

    def take_position():
        yield lambda p=st["pos"]: st["released"] >= p + 1 - nk
        st["pos"] += 1

    def tma():
        for it in range(n_tiles):
            for _ in range(nk):                                   # the Q landing takes every slot once
                yield lambda p=st["pos"]: st["released"] >= p + 1 - nk
                st["pos"] += 1
            st["q_loaded"] = it + 1
            vbase = it * nch

            def load_v(cv):
                yield lambda: st["pv"] >= vbase + cv - 1          # V buffer of chunk cv - 2 free
                st["v_loaded"] = vbase + cv + 1

            for pass_ in range(2):
                for c in range(0, nch, PAIR):
                    yield lambda p=st["pos"]: st["released"] >= p + 1 - nk
                    st["pos"] += 1
                    st["pairs_loaded"] += 1
                    if pass_ == 1:
                        for cc in range(c, c + PAIR):
                            if cc >= vlag:
                                yield from load_v(cc - vlag)
                if pass_ == 1:
                    for cv in range(max(0, nch - vlag), nch):
                        yield from load_v(cv)

    def prior():
        for g in range(n_tiles * nch):
            yield lambda g=g: st["pr_released"] >= g + 1 - npr
            st["pr_loaded"] = g + 1

    def mma():
        def issue():
            yield lambda: (st["pairs_loaded"] >= st["pairs_used"] + 1
                           and st["s_released"] >= st["s_issued"] + PAIR - nsb)
            st["pairs_used"] += 1
            st["s_issued"] += PAIR
            st["released"] += 1                                   # the pair's ring position, after its MMA

        for it in range(n_tiles):
            yield lambda it=it: st["q_loaded"] >= it + 1
            yield lambda: st["s_released"] >= st["s_issued"] + 1 - nsb   # drain buffer free
            st["released"] += nk                                   # the landing's positions
            for _ in range(0, nch, PAIR):
                yield from issue()
            nb = 0
            for c in range(nch):
                while nb < nch and nb + PAIR - 1 < c + nsb:
                    yield from issue()
                    nb += PAIR
                g = it * nch + c
                yield lambda g=g: st["p_staged"] >= g + 1 and st["v_loaded"] >= g + 1
                st["pv"] = g + 1
            st["ofull"] = it + 1

    def ew():
        s = 0
        for it in range(n_tiles):
            for c in range(0, nch, 2):
                yield lambda s=s: st["s_issued"] >= s + 2
                s += 2
                st["s_released"] = s
            for c in range(nch):
                g = it * nch + c
                yield lambda s=s, g=g: st["s_issued"] >= s + 1 and st["pr_loaded"] >= g + 1
                s += 1
                st["s_released"] = s
                st["pr_released"] = g + 1
                yield lambda g=g: st["pv"] >= g - 1
                st["p_staged"] = g + 1
            yield lambda it=it: st["ofull"] >= it + 1

    progs = [tma(), prior(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * len(progs)
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


# FwdCfg<true, DP> pooled (DP <= 128): (NK pair slots, NPR); V loads lag the K loads by NSB - 1 chunks
BF16_POOLED_FWD = {64: (3, 2), 128: (2, 2)}


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("nch", [2, 4, 6, 8, 16])
def test_forward_pooled_bf16_order_has_no_deadlock(D, nch):
    nk, npr = BF16_POOLED_FWD[D]
    assert _forward_pooled_bf16_order(nch, 3, nk, npr, NSB - 1) is None


@pytest.mark.parametrize("D", [64, 128])
def test_forward_pooled_bf16_v_lag_range(D):
    """Pass B's V(c) follows the K pair holding chunk c + VLAG, whose ring slot was last used by the pair NK pairs
    earlier and is free once that pair's score MMA is issued, i.e. once chunk c + VLAG - PAIR * NK + 1 < c + NSB is in
    flight: VLAG <= NSB + PAIR * NK - 2. Every lag from 0 to that bound runs (the kernel uses NSB - 1); the next one
    stops (the planted mistake is caught)."""
    nk, npr = BF16_POOLED_FWD[D]
    bound = NSB + PAIR * nk - 2
    sizes = (2, 4, 8, 16)
    for vlag in range(0, bound + 1):
        assert all(_forward_pooled_bf16_order(n, 3, nk, npr, vlag) is None for n in sizes), vlag
    assert _forward_pooled_bf16_order(16, 3, nk, npr, bound + 1) is not None


def _key_pass_pooled_f32_order(nch, n_tiles, nq, nsb, nst, slag, nr=2):
    """The pooled fp32 key pass with the dS scratch stores (geoattn_bwd_cols_kernel<false, 64, true>) over several
    tiles of one CTA as three cooperating programs (the prior is read from L2); returns None or the deadlock state.

    The K/V landing takes the query ring's next nq positions (each waits for the release of its previous use), the
    MMA warp copies K/V into tensor memory, drains the copies through a free score buffer and releases the nq
    positions; then per chunk the TMA warp loads Q/dO (the next ring position), the row records (nr ring) and stores
    the transposed dS tile of chunk c - slag once staged (the staging tile's second release). The MMA warp issues
    S^T/dP^T up to nsb chunks ahead and dV/dK per staged chunk (releasing its ring position and staging tile); the
    element-wise warps as in the bf16 model."""
    st = dict(pos=0, released=0, kv_loaded=0, q_loaded=0, rec_loaded=0, rec_released=0, s_issued=0, s_released=0,
              t_staged=0, t_mma=0, t_store=0, done=0)

    def tma():
        for it in range(n_tiles):
            for _ in range(nq):                                     # the landing takes every slot once
                yield lambda p=st["pos"]: st["released"] >= p + 1 - nq
                st["pos"] += 1
            st["kv_loaded"] = it + 1
            g0 = it * nch
            for c in range(nch):
                gc = g0 + c
                yield lambda p=st["pos"]: st["released"] >= p + 1 - nq
                st["pos"] += 1
                st["q_loaded"] = gc + 1
                yield lambda gc=gc: st["rec_released"] >= gc + 1 - nr
                st["rec_loaded"] = gc + 1
                if c >= slag:
                    yield lambda g=gc - slag: st["t_staged"] >= g + 1
                    st["t_store"] = gc - slag + 1
            for c in range(max(0, nch - slag), nch):
                yield lambda g=g0 + c: st["t_staged"] >= g + 1
                st["t_store"] = g0 + c + 1

    def mma():
        def issue(gc):
            yield lambda: st["q_loaded"] >= gc + 1 and st["s_released"] >= gc + 1 - nsb
            st["s_issued"] = gc + 1

        for it in range(n_tiles):
            g0 = it * nch
            yield lambda it=it: st["kv_loaded"] >= it + 1
            yield lambda g0=g0: st["s_released"] >= g0 + 1 - nsb      # the drain's score buffer
            st["released"] += nq
            yield from issue(g0)
            for c in range(nch):
                gc = g0 + c
                if nsb == 2 and c + 1 < nch:
                    yield from issue(gc + 1)
                yield lambda gc=gc: st["t_staged"] >= gc + 1
                st["t_mma"] = gc + 1
                st["released"] += 1
            st["done"] = it + 1

    def ew():
        for it in range(n_tiles):
            g0 = it * nch
            for c in range(nch):
                gc = g0 + c
                yield lambda gc=gc: st["s_issued"] >= gc + 1 and st["rec_loaded"] >= gc + 1
                st["s_released"] = st["rec_released"] = gc + 1
                yield lambda gc=gc: st["t_mma"] >= gc + 1 - nst and st["t_store"] >= gc + 1 - nst
                st["t_staged"] = gc + 1
            last = g0 + nch
            yield lambda it=it, last=last: st["done"] >= it + 1 and st["t_mma"] >= last and st["t_store"] >= last

    progs = [tma(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * len(progs)
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


# ColsCfg<false, 64, true>: NQ = 2, NSB = 2, NST = 2; the stores trail by SLAG = NQ - 1
@pytest.mark.parametrize("nch", [1, 2, 3, 8, 11, 16])
def test_key_pass_pooled_f32_store_lag_has_no_deadlock(nch):
    assert _key_pass_pooled_f32_order(nch, 4, 2, 2, 2, 1) is None


def test_key_pass_pooled_f32_store_lag_bound():
    """As in the bf16 key pass, a store lag up to NQ + NST - 1 runs and one more stops the pipeline."""
    nq, nsb, nst = 2, 2, 2
    bound = nq + nst - 1
    assert all(_key_pass_pooled_f32_order(n, 4, nq, nsb, nst, bound) is None for n in (1, 2, 3, 5, 8, 11, 16))
    assert _key_pass_pooled_f32_order(16, 4, nq, nsb, nst, bound + 1) is not None


def _forward_one_order(nch, n_tiles, nk, unit, pooled, nsb, npr):
    """The forward with a single score pass (geoattn_fwd_kernel<BF16, DP, true>) over several tiles as four
    cooperating programs; returns None or the deadlock state.

    Pass A only issues score MMAs: the TMA warp loads the K ring (nk slots; a slot holds `unit` chunks: one 64-key
    chunk in bf16, a pair of 32-key chunks in the pooled fp32 kernel), the MMA warp issues one score MMA per slot into
    `unit` of the nsb score buffers and releases the slot; the element-wise warps load two chunks' scores, release
    both buffers and keep the values in tensor memory. Pass B issues no score MMA: the TMA warp loads V per chunk (two
    buffers, each freed by its P.V MMA), the prior loader stages each chunk's prior tile (npr buffers), the
    element-wise warps stage P once the P.V two chunks back has run, and the MMA warp issues P.V per chunk. Q: bf16
    reloads it once the tile's last score MMA is issued; the pooled kernel lands it in the ring (nk positions,
    released after the copies and their drain through a free score buffer), possibly while the previous tile's pass B
    still runs."""
    st = dict(pos=0, released=0, q_loaded=0, q_released=0, k_loaded=0, k_used=0, v_loaded=0, pv=0, pr_loaded=0,
              pr_released=0, s_issued=0, s_released=0, p_staged=0, ofull=0)

    def tma():
        for it in range(n_tiles):
            if pooled:
                for _ in range(nk):
                    yield lambda p=st["pos"]: st["released"] >= p + 1 - nk
                    st["pos"] += 1
            else:
                yield lambda it=it: st["q_released"] >= it
            st["q_loaded"] = it + 1
            for _ in range(0, nch, unit):
                yield lambda p=st["pos"]: st["released"] >= p + 1 - nk
                st["pos"] += 1
                st["k_loaded"] += 1
            for c in range(nch):
                g = it * nch + c
                yield lambda g=g: st["pv"] >= g - 1
                st["v_loaded"] = g + 1

    def prior():
        for g in range(n_tiles * nch):
            yield lambda g=g: st["pr_released"] >= g + 1 - npr
            st["pr_loaded"] = g + 1

    def mma():
        for it in range(n_tiles):
            yield lambda it=it: st["q_loaded"] >= it + 1
            if pooled:
                yield lambda: st["s_released"] >= st["s_issued"] + 1 - nsb   # the drain's buffer
                st["released"] += nk
            for _ in range(0, nch, unit):
                yield lambda: (st["k_loaded"] >= st["k_used"] + 1
                               and st["s_released"] >= st["s_issued"] + unit - nsb)
                st["k_used"] += 1
                st["s_issued"] += unit
                st["released"] += 1
            if not pooled:
                st["q_released"] = it + 1
            for c in range(nch):
                g = it * nch + c
                yield lambda g=g: st["p_staged"] >= g + 1 and st["v_loaded"] >= g + 1
                st["pv"] = g + 1
            st["ofull"] = it + 1

    def ew():
        s = 0
        for it in range(n_tiles):
            for c in range(0, nch, 2):
                two = 2 if c + 1 < nch else 1
                yield lambda s=s, two=two: st["s_issued"] >= s + two
                s += two
                st["s_released"] = s
            for c in range(nch):
                g = it * nch + c
                yield lambda g=g: st["pr_loaded"] >= g + 1
                yield lambda g=g: st["pv"] >= g - 1
                st["p_staged"] = g + 1
                st["pr_released"] = g + 1
            yield lambda it=it: st["ofull"] >= it + 1

    progs = [tma(), prior(), mma(), ew()]
    waits = [next(p) for p in progs]
    done = [False] * len(progs)
    while not all(done):
        moved = False
        for i, prog in enumerate(progs):
            while not done[i] and waits[i]():
                try:
                    waits[i] = next(prog)
                except StopIteration:
                    done[i] = True
                moved = True
        if not moved:
            return dict(st)
    return None


@pytest.mark.parametrize("nch", [1, 2, 3, 5, 8])
def test_forward_one_bf16_order(nch):
    """FwdCfg<true, DP <= 128, true>: Q in shared memory, 3-deep ring of 64-key K chunks, two score buffers, two
    staged prior tiles; up to 8 chunks (512 keys), several tiles."""
    assert _forward_one_order(nch, 3, 3, 1, False, 2, 2) is None


@pytest.mark.parametrize("nch", [2, 4, 8, 16])
def test_forward_one_pooled_tf32_order(nch):
    """FwdCfg<false, 64, true>: Q pooled in tensor memory (its landing takes the 3-slot ring of K chunk pairs, even
    while the previous tile's pass B runs), one pair of 32-key score buffers; with a single score buffer a pair's MMA
    could never issue (the planted configuration stops)."""
    assert _forward_one_order(nch, 3, 3, 2, True, 2, 2) is None
    assert _forward_one_order(nch, 3, 3, 2, True, 1, 2) is not None
