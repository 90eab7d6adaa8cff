"""Dense GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).

Replaces the reference's register-fragment path for matmul kernels
(``compiler/mma.py``: ``RegFragment`` m16n8k16 fragments, ``LdmatrixLoad`` from
cp.async-filled shared memory, ``MmaSyncPtx``, ``RegStore``; ``compiler/coop.py``
``CpAsyncCopy``; ``compiler/memory.py`` swizzles).  The IR's matmul family
(``tests/problems/x_h_mm_1024`` and relatives) is recognised -- which buffer is A,
which is B and in which major order, the output and its dtype -- and lowered to
this template instead of emmy's 32x256 mma.sync schedule.

Kernel structure (one CTA per SM, persistent over output tiles):

* warp 0, lane 0 -- TMA producer: ``cp.async.bulk.tensor`` tiles of A (BM x 64 K,
  K-major) and B (64 K x BN, MN- or K-major) into a ``STAGES``-deep ring of
  128-byte-swizzled shared-memory stages, each guarded by a full/empty mbarrier pair;
* warp 1 -- allocates TMEM (two BN-column f32 accumulators); lane 0 issues
  ``tcgen05.mma.cta_group::1.kind::f16`` (M=128, N=BN, K=16) from shared-memory
  descriptors and ``tcgen05.commit``\\ s each stage back to the producer and each
  finished accumulator to the epilogue;
* warps 2-5 -- epilogue: ``tcgen05.ld.32x32b.x32`` (one accumulator row per
  thread), optional fused elementwise ops, ``cvt.rn.bf16x2.f32`` and 128-bit
  stores; the accumulator buffer is released as soon as it is read, so the next
  tile's MMAs overlap this tile's stores.

Tiles are walked in groups of 8 M-tiles so CTAs running together share A and B
panels in L2.  Every mbarrier wait is bounded (2 s of ``%globaltimer``): a stuck
pipeline records a status bit and the CTA releases its TMEM and exits.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from ..ptx import Ptx, entry, module
from .common import arg_params, load_pointer, param_symbol
from .tc import Waits, instr_desc, smem_desc_hi, smem_desc_lo_const

SMS = 148
GEMM_THREADS = 192       # warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
CONV_THREADS = 128       # warps 6-9 with 3xTF32 operands: the hi/lo split
ELEM_BYTES = {"bf16": 2, "f16": 2, "e4m3": 1, "f32": 4, "f64": 8}
AB_FORMAT = {"f16": 0, "bf16": 1, "e4m3": 0, "e5m2": 1, "f32": 2}   # f32 operands are read as tf32


@dataclass
class GemmConfig:
    M: int
    N: int
    K: int
    batch: int = 1
    ab: str = "bf16"              # operand type: bf16 | f16 | e4m3 | f32 (3xTF32, see split3)
    c: str = "bf16"               # output type: bf16 | f16 | f32
    b_kmajor: bool = False        # B stored [N, K] (else [K, N])
    BN: int = 256
    stages: int = 4
    acc_bufs: int = 2
    group_m: int = 16             # M tiles per raster group (the tiles in flight share A panels)
    serpentine: bool | None = None  # every other tile of a CTA walks K backwards (None: on
                                    # when TMA feeds the stages)
    pdl: bool = True                  # programmatic dependent launch: the prologue (barriers,
                                      # TMEM) overlaps the previous kernel's tail
    epilogue: tuple = ()          # ("relu",) | ("bias", buf) | ("residual", buf) | ("scale2", sa, sb)
    name: str = "k_gemm"
    a_param: str = "a"
    b_param: str = "b"
    c_param: str = "c"
    arg_params: list | None = None   # signature (meta.json arg_order) when compiled from IR
    buffers: tuple = ()              # pointer params to load (name list) for IR kernels
    pair: bool = False               # CTA pair (cta_group::2): 256-row tiles, B split by column
    operand_dtypes: tuple = ()       # (buffer, dtype) of epilogue operands
    ksplit: int = 0                  # K slices per tile (0: chosen from the shape; 1: none)
    tail_split: int = 0              # K slices of the tiles past the last full wave of CTAs / pairs
                                     # (0: chosen from the shape; 1: none)
    zero_slots: int = 0              # split-K partials: the full product goes to slice 0 of C and
    slot_stride: int = 0             # these many further slices (slot_stride elements apart) are zeroed
    operand_round: str | None = None  # f32 operands cast to "bf16" / "f16" before the product: one
                                      # exact tf32 MMA on the rounded values instead of 3xTF32
    direct: bool = False             # converter warps load A and B from global memory (rows that
    a_dtype: str = "f32"             # are not 16-byte aligned, 16-bit or mixed sources), with
    b_dtype: str = "f32"             # these element types, instead of TMA

    BM = 128                         # accumulator rows per CTA

    @property
    def MT(self) -> int:             # rows of one output tile
        return 256 if self.pair else 128

    @property
    def kind(self) -> str:
        return {"e4m3": "f8f6f4", "e5m2": "f8f6f4", "f32": "tf32"}.get(self.ab, "f16")

    @property
    def converts(self) -> bool:
        """f32 operands pass through the converter warps before the tf32 MMAs."""
        return self.ab == "f32"

    @property
    def split3(self) -> bool:
        """f32 operands: each is split into tf32 hi + lo parts in shared memory and the
        product accumulates hi*hi + hi*lo + lo*hi (three kind::tf32 MMAs per K step)."""
        return self.ab == "f32" and self.operand_round is None

    @property
    def BK(self) -> int:                 # K elements per stage: one 128-byte swizzle row
        return 128 // ELEM_BYTES[self.ab]

    @property
    def UK(self) -> int:                 # K per tcgen05.mma instruction (32 bytes)
        return 32 // ELEM_BYTES[self.ab]

    @property
    def tiles(self) -> tuple[int, int]:
        return -(-self.M // self.MT), -(-self.N // self.BN)


# Relative work rate of one SM per tile shape (bf16, 2048^3 .. 8192^3 on B200): a CTA
# pair's 256x256 tile halves each SM's shared-memory reads of B; a 128-wide N tile
# makes every MMA instruction re-read the whole A slice for half the columns.
_TILE_RATE = {("pair", 256): 1.05, (1, 256): 1.0, (1, 128): 0.75, (1, 64): 0.5}


def choose_bn(M: int, N: int, batch: int, min_bn: int = 64) -> int:
    """N tile width (<= 256) of single-CTA tiles: ``choose_tiling``'s estimate over
    the single-CTA shapes.  ``min_bn`` is the width of one 128-byte TMA box of an
    MN-major B (64 16-bit or 128 8-bit elements)."""
    return choose_tiling(M, N, batch, min_bn, pairs=False)["BN"]


# shared memory of the epilogue's store staging: per epilogue warp, its 32 rows x 32
# columns of 16-bit results, rows 80 bytes apart (64 bytes + 16 of padding: the rows' 16-byte
# pieces fall in distinct banks when each lane writes its own row)
EPI_ROW = 80
EPI_STAGE_BYTES = 4 * 32 * EPI_ROW


def _stages_fit(bn: int, cap: int = 8) -> int:
    """Stages of a 16-bit / 8-bit TMA ring that fit in shared memory beside the epilogue's
    staging: a stage holds one 128-byte K row of A (128 rows) and of B (bn columns).  Short
    K loops gain most from a deep ring (every K block of a 512^3 tile in flight: 5.2 us
    against 6.2 us with 4)."""
    stage = 128 * 128 + bn * 128
    return max(4, min(cap, (232448 - 256 - 1024 - EPI_STAGE_BYTES) // stage))


def choose_tiling(M: int, N: int, batch: int, min_bn: int = 64, pairs: bool = True) -> dict:
    """The tiling with the least estimated time: persistent waves over the SMs (or SM
    pairs) times one tile's MACs per SM divided by that shape's work rate.  Single
    CTAs run 128 x BN tiles (BN 256, 128 or 64) with as many stages as fit (4, 7 or 8),
    CTA pairs 256 x 256 tiles with 6 stages (M and N of 256 or more)."""
    cands = []
    if pairs and M >= 256 and N >= 256:
        tiles = batch * (-(-M // 256)) * (-(-N // 256))
        cands.append(((-(-tiles // (SMS // 2))) * 128 * 256 / _TILE_RATE[("pair", 256)],
                      0, {"pair": True, "BN": 256, "stages": 6}))
    for bn in (256, 128, 64):
        if bn < min_bn:
            continue
        tiles = batch * (-(-M // 128)) * (-(-N // bn))
        cands.append(((-(-tiles // SMS)) * 128 * bn / _TILE_RATE[(1, bn)], 1,
                      {"pair": False, "BN": bn, "stages": _stages_fit(bn)}))
    best = min(cands, key=lambda c: (c[0], c[1], -c[2]["BN"]))[2]
    if not best["pair"] and N < best["BN"]:
        bn = max(32, -(-N // 32) * 32)       # the epilogue reads TMEM 32 columns at a time
        bn = max(bn, min_bn)
        best = dict(best, BN=bn, stages=_stages_fit(bn))
    return best


def _tile_coords(p: Ptx, cfg: GemmConfig, t: str, ks: int = 1) -> tuple[str, str, str]:
    """Grouped raster: tile index -> (batch, m tile, n tile), all u32 registers.  With
    ``ks`` K slices per tile, ``t`` is a work unit: tile t / ks, slice t % ks.

    Tiles run M-fastest inside groups of ``group_m`` M tiles, so the tiles in flight at
    once (one per SM or SM pair) cover a block of group_m rows by a few columns, and the
    next wave moves along N over the same A panels.  With the serpentine K order (odd
    tiles of a CTA load K last to first) the next wave starts on the A slices the last
    one read most recently.  Measured at 8192^3 (CTA pairs, one launch): DRAM reads
    1047 MB with groups of 8 in K order, 853 MB with groups of 16 and the serpentine
    order (3.6 % less time in a power-capped run of 200 launches)."""
    if ks > 1:
        tt = p.reg("u32")
        p.emit(f"div.u32 {tt}, {t}, {ks}")
        t = tt
    tm, tn = cfg.tiles
    per_batch = tm * tn
    gsz = cfg.group_m * tn
    bt, r, g, first, gm, w, mt, nt = p.regs("u32", 8)
    p.emit(f"""
        div.u32 {bt}, {t}, {per_batch}
        rem.u32 {r}, {t}, {per_batch}
        div.u32 {g}, {r}, {gsz}
        mul.lo.u32 {first}, {g}, {cfg.group_m}
        sub.u32 {gm}, {tm}, {first}
        min.u32 {gm}, {gm}, {cfg.group_m}
        rem.u32 {w}, {r}, {gsz}
        rem.u32 {mt}, {w}, {gm}
        add.u32 {mt}, {mt}, {first}
        div.u32 {nt}, {w}, {gm}
    """)
    return bt, mt, nt


def choose_ksplit(cfg: GemmConfig, ntiles: int, kblocks: int, pair: bool) -> int:
    """K slices per tile when the tiles alone leave most SMs idle.  Splitting adds a fixed
    chain of about 5 us (the partial's stores, a GPU-scope fence, the ticket, the last
    slice's L2 reads), so it is taken only where it removes at least 8 K stages from the
    critical path of the converter-fed kernels (3xTF32 / direct loads, ~0.75 us a stage;
    a 16-bit TMA stage is ~0.15 us and never gains on B200, measured): the largest power of
    two that keeps the units within one wave, at least four K blocks per unit, and the
    last slice's reduction read (slices x one f32 tile) within 512 KB."""
    if cfg.ksplit:
        return cfg.ksplit
    if pair or cfg.zero_slots or not cfg.converts or 2 * ntiles > SMS:
        return 1
    ks = 1
    while (ntiles * ks * 2 <= SMS and kblocks % (ks * 2) == 0 and kblocks // (ks * 2) >= 4
           and ks * 2 * cfg.MT * cfg.BN * 4 <= 512 * 1024):
        ks *= 2
    return ks if kblocks - kblocks // ks >= 8 else 1


def choose_tail_split(cfg: GemmConfig, ntiles: int, kblocks: int, workers: int) -> int:
    """K slices for the tiles of the last, partial wave (the tail), when whole tiles would
    leave workers (SMs or SM pairs) idle in it.  The first (ntiles // workers) waves run
    whole tiles; the R tiles left are cut into ts slices each and spread over the workers,
    so the tail takes ceil(R ts / workers) / ts of a tile's time instead of a whole one.
    Each sliced unit writes its f32 partial to a workspace and the last slice of a tile
    (a ticket per warp quarter) sums them in slice order, as with ``ksplit``.  Taken when
    it saves at least 4 % of the kernel's time (4096 x 14336 x 4096 on one B200: 896 pair
    tiles = 12 full waves + 8 tiles, which 8 slices each spread over 64 pairs)."""
    if cfg.tail_split:
        return cfg.tail_split
    if cfg.converts or cfg.zero_slots or cfg.ksplit > 1 or cfg.direct:
        return 1
    full, rem = divmod(ntiles, workers)
    if full == 0 or rem == 0:
        return 1
    # a tile's time at the tensor rate (7736 flop / clock / SM at ~1.9 GHz) against the
    # fix-up: every unit writes its f32 partial, the finishing slice reads all of them
    # (about 300 GB/s per SM pair, 150 GB/s per SM)
    sms = 2 if cfg.pair else 1
    tile_s = 2.0 * cfg.MT * cfg.BN * cfg.K / (sms * 7736 * 1.9e9)
    part = cfg.MT * cfg.BN * 4
    best, best_t = 1, 1.0
    for ts in (2, 4):
        if kblocks % ts or kblocks // ts < 4 or rem * ts * part > 256 * 2 ** 20:
            continue
        if ts > 2 and cfg.K > 4096:
            # measured on pair tiles: 4 slices of 8192-deep tiles lose (8192 x 1024 x 8192:
            # 97 -> 130 us) where the estimate says they gain; 4 slices of 4096 gain 2-3 %
            continue
        fix = (part + ts * part) / (sms * 150e9) / tile_s
        t = -(-rem * ts // workers) / ts + fix
        if t < best_t - 1e-9:
            best, best_t = ts, t
    return best if (1.0 - best_t) / (full + 1) >= 0.04 else 1


def _unit_plan(p: Ptx, cfg: GemmConfig, t: str, ks: int, kps: int, tail):
    """Work unit t -> (batch, m tile, n tile, first K block, K blocks, sliced pred, tail unit).

    Without a tail split: unit t is slice t % ks of tile t / ks (ks uniform K slices, kps
    blocks each).  With ``tail = (D, ts, kpt)``: units below D are whole tiles (kps blocks),
    unit D + v is slice v % ts (kpt blocks) of tile D + v / ts."""
    if tail is None:
        bt, mt, nt = _tile_coords(p, cfg, t, ks)
        kb0 = p.reg("u32")
        p.emit(f"rem.u32 {kb0}, {t}, {ks}\nmul.lo.u32 {kb0}, {kb0}, {kps}")
        return bt, mt, nt, kb0, str(kps), None, None
    D, ts, kpt = tail
    tile, kb0, nkb, v, sl = p.regs("u32", 5)
    psl = p.reg("pred")
    p.emit(f"""
        setp.ge.u32 {psl}, {t}, {D}
        mov.u32 {tile}, {t}
        mov.u32 {kb0}, 0
        mov.u32 {nkb}, {kps}
        sub.u32 {v}, {t}, {D}
        @{psl} div.u32 {tile}, {v}, {ts}
        @{psl} add.u32 {tile}, {tile}, {D}
        @{psl} rem.u32 {sl}, {v}, {ts}
        @{psl} mul.lo.u32 {kb0}, {sl}, {kpt}
        @{psl} mov.u32 {nkb}, {kpt}
    """)
    bt, mt, nt = _tile_coords(p, cfg, tile, 1)
    return bt, mt, nt, kb0, nkb, psl, v


def _emit_zero_slices(p: Ptx, cfg: GemmConfig, cptr: str, tid: str, nthreads: int) -> None:
    """Split-K partial slices 1 .. zero_slots of C (the whole product goes to slice 0) are
    one contiguous range; every thread of the grid zeroes part of it with coalesced
    stores before the roles start (16-byte stores when the slices are whole float4s)."""
    w = 4 if cfg.slot_stride % 4 == 0 else 1
    units = cfg.zero_slots * cfg.slot_stride // w
    gi, gs, a = p.reg("u32"), p.reg("u32"), p.reg("b64")
    pz = p.reg("pred")
    top, done = p.label("zero_slices"), p.label("zero_done")
    zero = "{0f00000000, 0f00000000, 0f00000000, 0f00000000}" if w == 4 else "0f00000000"
    p.emit(f"""
        mov.u32 {gi}, %ctaid.x
        mad.lo.u32 {gi}, {gi}, {nthreads}, {tid}
        mov.u32 {gs}, %nctaid.x
        mul.lo.u32 {gs}, {gs}, {nthreads}
    """)
    p.place(top)
    p.emit(f"""
        setp.ge.u32 {pz}, {gi}, {units}
        @{pz} bra {done}
        mul.wide.u32 {a}, {gi}, {4 * w}
        add.s64 {a}, {a}, {cptr}
        st.global{'.v4' if w == 4 else ''}.f32 [{a}+{cfg.slot_stride * 4}], {zero}
        add.u32 {gi}, {gi}, {gs}
        bra {top}
    """)
    p.place(done)


def emit_gemm_module(cfg: GemmConfig) -> str:
    p = Ptx()
    split, conv = cfg.split3, cfg.converts
    M, N, K, BM, BN, BK, S = cfg.M, cfg.N, cfg.K, cfg.BM, cfg.BN, cfg.BK, cfg.stages
    eb = ELEM_BYTES[cfg.ab]
    cb = ELEM_BYTES[cfg.c]
    tm, tn = cfg.tiles
    ntiles = cfg.batch * tm * tn
    kblocks = -(-K // BK)
    pair = cfg.pair
    KS = choose_ksplit(cfg, ntiles, kblocks, pair)
    if KS > 1 and (pair or kblocks % KS):
        raise NotImplementedError("K slices need 1-CTA tiles and whole K blocks per slice")
    kps, nunits = kblocks // KS, ntiles * KS
    workers = SMS // 2 if pair else SMS
    TS = choose_tail_split(cfg, ntiles, kblocks, workers) if KS == 1 else 1
    tail = None
    if TS > 1:
        if kblocks % TS or cfg.direct or cfg.converts:
            raise NotImplementedError("tail K slices need whole K blocks and TMA-fed operands")
        D = (ntiles // workers) * workers
        tail = (D, TS, kblocks // TS)
        nunits = D + (ntiles - D) * TS
    BNc = BN // 2 if pair else BN           # B columns held by one CTA
    a_bytes = BM * BK * eb                  # 16 KB
    b_bytes = BNc * BK * eb                 # 32 KB at BN = 256 (16 KB per CTA of a pair)
    raw_bytes = a_bytes + b_bytes           # what the TMA copies write per stage and CTA
    if conv and pair:
        raise NotImplementedError("converted f32 operands on CTA pairs")
    # 3xTF32: the stage holds the tf32 hi parts (in place of the loaded f32 values)
    # followed by the lo parts
    stage_bytes = raw_bytes * (2 if split else 1)
    ncols = max(32, 1 << math.ceil(math.log2(BN * cfg.acc_bufs)))
    if ncols > 512:
        raise NotImplementedError("accumulators exceed TMEM")
    smem = S * stage_bytes + 1024           # +1 KB to align the ring to 1024 B
    if smem > 232448 - 256:
        raise NotImplementedError("stage ring exceeds shared memory")
    # 16-bit results leave through shared memory (see _emit_epilogue) when it has room
    epi_off = None
    if cfg.c in ("bf16", "f16") and N % 8 == 0 and smem + EPI_STAGE_BYTES <= 232448 - 256:
        epi_off = S * stage_bytes
        smem += EPI_STAGE_BYTES
    # tf32 operands read MN-major need the 32-byte-atom swizzle; the 3xTF32 converter writes
    # B K-major instead (the layout A has), so the MMAs read both operands K-major
    mma_b_kmajor = cfg.b_kmajor or cfg.converts
    idesc = instr_desc(cfg.MT, BN, AB_FORMAT[cfg.ab], AB_FORMAT[cfg.ab], False, not mma_b_kmajor)
    cg = "cta_group::2" if pair else "cta_group::1"
    a_hi = smem_desc_hi(1024)
    a_lo = smem_desc_lo_const(16)
    if mma_b_kmajor:
        b_hi, b_lo = smem_desc_hi(1024), smem_desc_lo_const(16)
    else:
        # MN-major: 64-element (128-byte) column blocks of BK K-rows each, BK*128 bytes apart
        b_hi, b_lo = smem_desc_hi(1024), smem_desc_lo_const(BK * 128)
    nb_mn = BNc // (128 // eb)              # MN-major B: number of 128-byte column blocks
    if not cfg.b_kmajor and BNc % (128 // eb):
        raise NotImplementedError(f"BN={BN} is not a whole number of 128-byte B boxes")
    rank = 3 if cfg.batch > 1 else 2

    p.comment(f"tcgen05 GEMM {cfg.batch}x{M}x{N}x{K} {cfg.ab}->{cfg.c}, tile {cfg.MT}x{BN}x{BK}"
              f"{' on a CTA pair (cta_group::2)' if pair else ''}, "
              f"{S} stages, {cfg.acc_bufs} TMEM accumulators, B {'K' if cfg.b_kmajor else 'MN'}-major")
    # ---------------------------------------------------------------- setup
    ptr = {}
    for name in cfg.buffers:
        ptr[name] = load_pointer(p, name)
    status = p.reg("b64")
    p.emit(f"ld.param.u64 {status}, [param__status]\ncvta.to.global.u64 {status}, {status}")
    direct = cfg.direct
    if direct and not conv:
        raise NotImplementedError("direct operand loads need the converter warps")
    tma_a, tma_b = p.reg("b64"), p.reg("b64")
    if not direct:
        p.emit(f"""
            mov.u64 {tma_a}, param__tmap_a
            cvta.param.u64 {tma_a}, {tma_a}
            mov.u64 {tma_b}, param__tmap_b
            cvta.param.u64 {tma_b}, {tma_b}
        """)
    tid, warp, lane = p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mov.u32 {tid}, %tid.x
        shr.u32 {warp}, {tid}, 5
        and.b32 {lane}, {tid}, 31
    """)
    if cfg.pdl:
        # the next kernel of the stream may start its own prologue now (it waits for this
        # one before touching global memory, like this one below)
        p.emit("griddepcontrol.launch_dependents")
    if cfg.zero_slots:
        if cfg.pdl:
            p.emit("griddepcontrol.wait")
        _emit_zero_slices(p, cfg, ptr[cfg.c_param], tid, GEMM_THREADS + (CONV_THREADS if conv else 0))
    ring, bars, abort, tslot = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mov.u32 {ring}, dsmem
        add.u32 {ring}, {ring}, 1023
        and.b32 {ring}, {ring}, -1024
        mov.u32 {bars}, gbars
        mov.u32 {abort}, gabort
        mov.u32 {tslot}, gtmem
    """)
    # barrier layout: full[S], empty[S], tfull[A], tempty[A]
    # ... and with 3xTF32 conv[S]: the stage's hi/lo parts are written
    # and cread: every converter has read the stage's B before any overwrites it
    nbar = 2 * S + 2 * cfg.acc_bufs + (S + 1 if conv else 0)
    full0, empty0, tfull0, tempty0 = 0, 8 * S, 16 * S, 16 * S + 8 * cfg.acc_bufs
    conv0 = 16 * S + 16 * cfg.acc_bufs
    cread = conv0 + 8 * S
    p0 = p.reg("pred")
    init_done = p.label("init_done")
    p.emit(f"setp.ne.u32 {p0}, {tid}, 0\n@{p0} bra {init_done}")
    for s in range(S):
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{full0 + 8 * s}], 1")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{empty0 + 8 * s}], 1")
    for b in range(cfg.acc_bufs):
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{tfull0 + 8 * b}], 1")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{tempty0 + 8 * b}], {256 if pair else 128}")
    if conv:
        for st in range(S + 1):
            p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{conv0 + 8 * st}], {CONV_THREADS}")
    p.emit(f"st.shared.u32 [{abort}], 0\nfence.mbarrier_init.release.cluster\nfence.proxy.async.shared::cta")
    p.place(init_done)
    crank, lfull, ltempty = p.reg("u32"), p.reg("u32"), p.reg("u32")
    pleader = p.reg("pred")
    if pair:
        # both CTAs' barriers are initialised before either CTA touches its peer's
        p.emit(f"""
            barrier.cluster.arrive.release
            barrier.cluster.wait.acquire
            mov.u32 {crank}, %cluster_ctarank
            setp.eq.u32 {pleader}, {crank}, 0
            add.u32 {lfull}, {bars}, {full0}
            mapa.shared::cluster.u32 {lfull}, {lfull}, 0
            add.u32 {ltempty}, {bars}, {tempty0}
            mapa.shared::cluster.u32 {ltempty}, {ltempty}, 0
        """)
    # TMEM allocation by warp 1 (warp-collective; both CTAs of a pair)
    p1 = p.reg("pred")
    alloc_done = p.label("alloc_done")
    p.emit(f"setp.ne.u32 {p1}, {warp}, 1\n@{p1} bra {alloc_done}")
    p.emit(f"""
        tcgen05.alloc.{cg}.sync.aligned.shared::cta.b32 [{tslot}], {ncols}
        tcgen05.relinquish_alloc_permit.{cg}.sync.aligned
    """)
    p.place(alloc_done)
    if cfg.pdl and not cfg.zero_slots:
        # every role waits for the stream's previous kernel (complete, its writes visible)
        # before its first global load or store; barrier set-up and the TMEM allocation
        # above ran while that kernel finished
        p.emit("griddepcontrol.wait")
    tbase = p.reg("u32")
    p.emit(f"""
        tcgen05.fence::before_thread_sync
        barrier.sync 0
        tcgen05.fence::after_thread_sync
        ld.shared.u32 {tbase}, [{tslot}]
    """)
    waits = Waits(p, status, abort)
    finish = p.label("finish")
    cta, nct = p.reg("u32"), p.reg("u32")
    if pair:    # tiles are walked per cluster
        p.emit(f"mov.u32 {cta}, %clusterid.x\nmov.u32 {nct}, %nclusterid.x")
    else:
        p.emit(f"mov.u32 {cta}, %ctaid.x\nmov.u32 {nct}, %nctaid.x")

    # ------------------------------------------------------------ producer
    role_mma, role_epi = p.label("role_mma"), p.label("role_epi")
    pr = p.reg("pred")
    p.emit(f"setp.ne.u32 {pr}, {warp}, 0\n@{pr} bra {role_mma}")
    pl = p.reg("pred")
    p.emit(f"setp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")
    if direct:      # the converter warps fetch the operands themselves
        p.emit(f"bra {finish}")
    p.emit(f"prefetch.tensormap [{tma_a}]\nprefetch.tensormap [{tma_b}]")
    t, s, ph = p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {t}, {cta}\nmov.u32 {s}, 0\nmov.u32 {ph}, 0")
    rev = None
    if cfg.serpentine or (cfg.serpentine is None and not direct):
        # the CTA's odd-numbered tiles load their K blocks last to first: the tiles of the
        # next wave then start on the operand slices the last wave read most recently
        rev = p.reg("pred")
        p.emit(f"setp.ne.u32 {rev}, {cta}, {cta}")
    tl, td = p.label("p_tile"), p.label("p_done")
    p.place(tl)
    pt = p.reg("pred")
    p.emit(f"setp.ge.u32 {pt}, {t}, {nunits}\n@{pt} bra {td}")
    # the unit's tile, first K block and number of K blocks
    bt, mt, nt, kb0, nkb, _, _ = _unit_plan(p, cfg, t, KS, kps, tail)
    m0, n0 = p.reg("u32"), p.reg("u32")
    p.emit(f"mul.lo.u32 {m0}, {mt}, {cfg.MT}\nmul.lo.u32 {n0}, {nt}, {BN}")
    if pair:    # this CTA's rows of the 256-row tile and its half of the B columns
        p.emit(f"mad.lo.u32 {m0}, {crank}, {BM}, {m0}\nmad.lo.u32 {n0}, {crank}, {BNc}, {n0}")
    kb, kx = p.reg("u32"), p.reg("u32")
    kl = p.label("p_k")
    p.emit(f"mov.u32 {kb}, 0")
    p.place(kl)
    eaddr, faddr, sa, sbb, par = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {eaddr}, {s}, 8, {bars}
        add.u32 {faddr}, {eaddr}, {full0}
        add.u32 {eaddr}, {eaddr}, {empty0}
        xor.b32 {par}, {ph}, 1
    """)
    waits.wait(eaddr, par, "producer", finish)
    if pair:
        # both CTAs' copies complete on the leader's full barrier; only the leader
        # announces the stage's bytes (both halves)
        p.emit(f"""
            @{pleader} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{faddr}], {2 * raw_bytes}
            mad.lo.u32 {faddr}, {s}, 8, {lfull}
        """)
        tma = "cp.async.bulk.tensor.{r}d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
    else:
        p.emit(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{faddr}], {raw_bytes}")
        tma = "cp.async.bulk.tensor.{r}d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
    tma = tma.format(r=rank)
    p.emit(f"""
        mad.lo.u32 {sa}, {s}, {stage_bytes}, {ring}
        add.u32 {sbb}, {sa}, {a_bytes}
        add.u32 {kx}, {kb}, {kb0}
    """)
    if rev is not None:
        if tail is None:
            p.emit(f"@{rev} sub.u32 {kx}, {kps - 1}, {kb}\n@{rev} add.u32 {kx}, {kx}, {kb0}")
        else:
            p.emit(f"@{rev} sub.u32 {kx}, {nkb}, 1\n@{rev} sub.u32 {kx}, {kx}, {kb}\n"
                   f"@{rev} add.u32 {kx}, {kx}, {kb0}")
    p.emit(f"mul.lo.u32 {kx}, {kx}, {BK}")
    zc = f", {bt}" if rank == 3 else ""
    p.emit(f"{tma} [{sa}], [{tma_a}, {{{kx}, {m0}{zc}}}], [{faddr}]")
    if cfg.b_kmajor:
        p.emit(f"{tma} [{sbb}], [{tma_b}, {{{kx}, {n0}{zc}}}], [{faddr}]")
    else:
        blk = 128 // eb                      # 64 bf16 / 128 fp8 columns per box
        for j in range(nb_mn):
            nx, dst = p.reg("u32"), p.reg("u32")
            p.emit(f"add.u32 {nx}, {n0}, {j * blk}\nadd.u32 {dst}, {sbb}, {j * BK * 128}")
            p.emit(f"{tma} [{dst}], [{tma_b}, {{{nx}, {kx}{zc}}}], [{faddr}]")
    ps = p.reg("pred")
    p.emit(f"""
        add.u32 {s}, {s}, 1
        setp.eq.u32 {ps}, {s}, {S}
        @{ps} mov.u32 {s}, 0
        @{ps} xor.b32 {ph}, {ph}, 1
        add.u32 {kb}, {kb}, 1
        setp.lt.u32 {ps}, {kb}, {nkb}
        @{ps} bra {kl}
        add.u32 {t}, {t}, {nct}
    """)
    if rev is not None:
        p.emit(f"not.pred {rev}, {rev}")
    p.emit(f"bra {tl}")
    p.place(td)
    p.emit(f"bra {finish}")

    # ----------------------------------------------------------------- MMA
    p.place(role_mma)
    p.emit(f"setp.ne.u32 {pr}, {warp}, 1\n@{pr} bra {role_epi}")
    p.emit(f"setp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")
    if pair:
        p.emit(f"@!{pleader} bra {finish}")
        mask = p.reg("b16")
        p.emit(f"mov.b16 {mask}, 3")
        commit = ("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster"
                  ".multicast::cluster.b64 [{a}], " + mask)
    else:
        commit = "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{a}]"
    t2, s2, ph2, tc = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {t2}, {cta}\nmov.u32 {s2}, 0\nmov.u32 {ph2}, 0\nmov.u32 {tc}, 0")
    ml, md = p.label("m_tile"), p.label("m_done")
    p.place(ml)
    p.emit(f"setp.ge.u32 {pt}, {t2}, {nunits}\n@{pt} bra {md}")
    ab, aph, tea, tfa, dt = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        rem.u32 {ab}, {tc}, {cfg.acc_bufs}
        div.u32 {aph}, {tc}, {cfg.acc_bufs}
        and.b32 {aph}, {aph}, 1
        xor.b32 {aph}, {aph}, 1
        mad.lo.u32 {tea}, {ab}, 8, {bars}
        add.u32 {tfa}, {tea}, {tfull0}
        add.u32 {tea}, {tea}, {tempty0}
        mad.lo.u32 {dt}, {ab}, {BN}, {tbase}
    """)
    waits.wait(tea, aph, "mma", finish)
    p.emit("tcgen05.fence::after_thread_sync")
    nkb2 = str(kps)
    if tail is not None:           # a sliced tail unit runs kpt K blocks
        nkb2 = p.reg("u32")
        ptl = p.reg("pred")
        p.emit(f"setp.ge.u32 {ptl}, {t2}, {tail[0]}\nselp.u32 {nkb2}, {tail[2]}, {kps}, {ptl}")
    kb2 = p.reg("u32")
    mk = p.label("m_k")
    p.emit(f"mov.u32 {kb2}, 0")
    p.place(mk)
    fa2, ea2 = p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {fa2}, {s2}, 8, {bars}
        add.u32 {ea2}, {fa2}, {empty0}
        add.u32 {fa2}, {fa2}, {conv0 if conv else full0}
    """)
    waits.wait(fa2, ph2, "mma", finish)
    p.emit("tcgen05.fence::after_thread_sync")
    sa2, sb2 = p.reg("u32"), p.reg("u32")
    p.emit(f"mad.lo.u32 {sa2}, {s2}, {stage_bytes}, {ring}\nadd.u32 {sb2}, {sa2}, {a_bytes}")
    # operand pairs per K step: (A, B), or with 3xTF32 (A hi, B hi), (A hi, B lo), (A lo, B hi)
    pairs_ab = [(0, 0), (0, raw_bytes), (raw_bytes, 0)] if split else [(0, 0)]
    for kk in range(BK // cfg.UK):
        a_off = kk * 32                                   # 32 bytes of K inside the swizzle row
        b_off = kk * 32 if mma_b_kmajor else kk * (cfg.UK * 128)   # MN-major: UK K-rows of 128 B
        for j, (ax, bx) in enumerate(pairs_ab):
            alo, blo, ad, bd = p.reg("u32"), p.reg("u32"), p.reg("b64"), p.reg("b64")
            pacc = p.reg("pred")
            p.emit(f"""
                add.u32 {alo}, {sa2}, {a_off + ax}
                shr.u32 {alo}, {alo}, 4
                or.b32 {alo}, {alo}, {a_lo}
                mov.b64 {ad}, {{{alo}, {a_hi}}}
                add.u32 {blo}, {sb2}, {b_off + bx}
                shr.u32 {blo}, {blo}, 4
                or.b32 {blo}, {blo}, {b_lo}
                mov.b64 {bd}, {{{blo}, {b_hi}}}
            """)
            if kk == 0 and j == 0:
                p.emit(f"setp.ne.u32 {pacc}, {kb2}, 0")
            else:
                p.emit(f"setp.eq.u32 {pacc}, {kb2}, {kb2}")
            p.emit(f"tcgen05.mma.{cg}.kind::{cfg.kind} [{dt}], {ad}, {bd}, {idesc}, {pacc}")
    p.emit(commit.format(a=ea2))
    p.emit(f"""
        add.u32 {s2}, {s2}, 1
        setp.eq.u32 {ps}, {s2}, {S}
        @{ps} mov.u32 {s2}, 0
        @{ps} xor.b32 {ph2}, {ph2}, 1
        add.u32 {kb2}, {kb2}, 1
        setp.lt.u32 {ps}, {kb2}, {nkb2}
        @{ps} bra {mk}
        {commit.format(a=tfa)}
        add.u32 {tc}, {tc}, 1
        add.u32 {t2}, {t2}, {nct}
        bra {ml}
    """)
    p.place(md)
    p.emit(f"bra {finish}")

    # ------------------------------------------------------------ epilogue
    p.place(role_epi)
    if conv:
        role_conv = p.label("role_conv")
        p.emit(f"setp.ge.u32 {pr}, {warp}, {GEMM_THREADS // 32}\n@{pr} bra {role_conv}")
    _emit_epilogue(p, cfg, ptr, bars, tfull0, tempty0, tbase, warp, lane, cta, nct, nunits,
                   waits, finish, crank if pair else None, ltempty if pair else None, KS, tail,
                   None if epi_off is None else (ring, epi_off))
    if conv:
        p.place(role_conv)
        if direct:
            _emit_direct_loader(p, cfg, ptr, tid, ring, bars, empty0, conv0, a_bytes, raw_bytes,
                                stage_bytes, kps, cta, nct, nunits, waits, finish, KS)
        else:
            _emit_split_tf32(p, cfg, tid, ring, bars, full0, conv0, cread, a_bytes, raw_bytes,
                             stage_bytes, kps, cta, nct, nunits, waits, finish)

    # -------------------------------------------------------------- finish
    p.place(finish)
    pw1 = p.reg("pred")
    done = p.label("done")
    p.emit(f"""
        tcgen05.fence::before_thread_sync
        barrier.sync 0
    """)
    if pair:    # neither CTA leaves while its peer may still use its smem, TMEM or barriers
        p.emit("barrier.cluster.arrive.release\nbarrier.cluster.wait.acquire")
    p.emit(f"""
        tcgen05.fence::after_thread_sync
        setp.ne.u32 {pw1}, {warp}, 1
        @{pw1} bra {done}
        bar.warp.sync -1
        tcgen05.dealloc.{cg}.sync.aligned.b32 {tbase}, {ncols}
    """)
    p.place(done)
    p.emit("ret")

    params = list(cfg.arg_params or [f".param .u64 {param_symbol(n)}" for n in cfg.buffers])
    if not direct:
        params += [".param .align 64 .b8 param__tmap_a[128]", ".param .align 64 .b8 param__tmap_b[128]"]
    if KS > 1 or tail is not None:
        params += [".param .u64 param__ksplit_ws", ".param .u64 param__ksplit_tickets"]
    params += [".param .u64 param__status"]
    nthreads = GEMM_THREADS + (CONV_THREADS if conv else 0)
    # one CTA per SM (its shared memory allows no more): registers are not scarce, so
    # let the allocator keep the epilogue's rows in registers instead of spilling
    text = entry(cfg.name, params, p, maxntid=nthreads, extra_directives="\n.maxnreg 128")
    statics = (f"\t.shared .align 8 .b64 gbars[{nbar}];\n\t.shared .align 4 .u32 gabort;\n"
               f"\t.shared .align 4 .u32 gtmem;\n")
    text = text.replace("{\n", "{\n" + statics, 1)
    grid = 2 * min(ntiles, SMS // 2) if pair else min(nunits, SMS)
    a_dims = [K, M] + ([cfg.batch] if rank == 3 else [])
    a_str = [K * eb] + ([M * K * eb] if rank == 3 else [])
    if cfg.b_kmajor:
        b_dims = [K, N] + ([cfg.batch] if rank == 3 else [])
        b_str = [K * eb] + ([N * K * eb] if rank == 3 else [])
        b_box = [BK, BNc] + ([1] if rank == 3 else [])
    else:
        b_dims = [N, K] + ([cfg.batch] if rank == 3 else [])
        b_str = [N * eb] + ([N * K * eb] if rank == 3 else [])
        b_box = [128 // eb, BK] + ([1] if rank == 3 else [])
    launch = {
        "kind": "gemm", "grid": [grid, 1, 1], "block": [nthreads, 1, 1], "cluster": [2 if pair else 1, 1, 1],
        "smem": smem, "flops": 2 * cfg.batch * M * N * K, "tiles": ntiles, "ksplit": KS,
        "tail_split": TS, "tail_tiles": 0 if tail is None else ntiles - tail[0],
        "pdl": bool(cfg.pdl),
        "extra_params": ([] if direct else [
            {"kind": "tmap", "buffer": cfg.a_param, "dtype": cfg.ab, "dims": a_dims, "strides": a_str,
             "box": [BK, BM] + ([1] if rank == 3 else []), "swizzle": 128},
            {"kind": "tmap", "buffer": cfg.b_param, "dtype": cfg.ab, "dims": b_dims, "strides": b_str,
             "box": b_box, "swizzle": 128},
        ]) + ([{"kind": "scratch", "bytes": nunits * cfg.MT * BN * 4},
               {"kind": "scratch", "bytes": ntiles * 4 * 4}] if KS > 1 else []) +
        ([{"kind": "scratch", "bytes": (nunits - tail[0]) * cfg.MT * BN * 4},
          {"kind": "scratch", "bytes": (ntiles - tail[0]) * 2 * 4 * 4}] if tail is not None else []) +
        [{"kind": "status"}],
    }
    return module([text], launch, globals_=[".extern .shared .align 1024 .b8 dsmem[];"])


def _tf32_round(p: Ptx, x: str, mode: str) -> str:
    """x rounded to bf16 / f16 (nearest even, as the IR's cast), as an f32 bit pattern: a
    value a tf32 operand holds exactly, so the MMA's products are the 16-bit products."""
    if mode not in ("bf16", "f16"):
        raise NotImplementedError(f"operand rounding to {mode}")
    h, r = p.reg("b16"), p.reg("b32")
    if mode == "bf16":
        z = p.reg("b16")
        p.emit(f"cvt.rn.bf16.f32 {h}, {x}\nmov.b16 {z}, 0\nmov.b32 {r}, {{{z}, {h}}}")
    else:
        p.emit(f"cvt.rn.f16.f32 {h}, {x}\ncvt.f32.f16 {r}, {h}")
    return r


def _tf32_split(p: Ptx, x: str) -> tuple[str, str]:
    """hi = tf32(x), lo = tf32(x - hi), both as f32 bit patterns with the low 13 bits clear."""
    hi, lo = p.reg("b32"), p.reg("b32")
    p.emit(f"""
        cvt.rna.tf32.f32 {hi}, {x}
        and.b32 {hi}, {hi}, -8192
        sub.rn.f32 {lo}, {x}, {hi}
        cvt.rna.tf32.f32 {lo}, {lo}
        and.b32 {lo}, {lo}, -8192
    """)
    return hi, lo


def _convert(p: Ptx, cfg: GemmConfig, xs: list) -> list:
    """(hi, lo) per value: the 3xTF32 split, or (rounded, None) for cast operands."""
    if cfg.operand_round:
        return [(_tf32_round(p, x, cfg.operand_round), None) for x in xs]
    return [_tf32_split(p, x) for x in xs]


def _emit_split_tf32(p: Ptx, cfg: GemmConfig, tid, ring, bars, full0, conv0, cread, a_bytes, raw_bytes,
                     stage_bytes, kblocks, cta, nct, ntiles, waits: Waits, finish: str) -> None:
    """Converter warps of the 3xTF32 GEMM.  Once a stage's f32 tiles have landed, each
    value x becomes hi = tf32(x) and lo = tf32(x - hi), both exact tf32 values, so the
    tensor core's reading of tf32 operands adds no rounding of its own, and
    hi*hi + hi*lo + lo*hi misses x*y by the lo*lo term and the rounding of lo: about
    2^-21 relative per product.  hi replaces x; lo goes ``raw_bytes`` further on.

    A (K-major, and B when stored [N, K]) is split element by element: the 128-byte
    swizzle is kept as it is.  An MN-major B tile (32-column blocks of BK K-rows, as the
    TMA boxes land) is transposed on the way into the K-major layout A has, because
    tf32 operands read MN-major need the 32-byte-atom swizzle: every converter reads
    its values first and arrives on ``cread``; after that barrier's (bounded) wait the
    transposed hi values overwrite the raw tile.  Generic-proxy stores are made visible
    to the tensor core (async proxy) by ``fence.proxy.async`` before the arrival on
    conv[stage] that the MMA warp waits for.  Operands the IR casts to bf16 / f16 are
    rounded instead (``operand_round``): one value, no lo part, one MMA per K step."""
    BK, BNc = cfg.BK, cfg.BN
    ctid = p.reg("u32")
    p.emit(f"sub.u32 {ctid}, {tid}, {GEMM_THREADS}")
    flat = raw_bytes if cfg.b_kmajor else a_bytes     # bytes split element by element
    per = flat // 16 // CONV_THREADS                   # 16-byte vectors per thread and stage
    assert flat % (16 * CONV_THREADS) == 0
    rd, wr = [], []
    if not cfg.b_kmajor:
        # (row n of the K-major tile, 16-byte K chunk c) items; n fastest across threads
        assert BNc & (BNc - 1) == 0 and BNc >= 32 and (BNc * (BK // 4)) % CONV_THREADS == 0
        lg = BNc.bit_length() - 1
        for j in range(BNc * (BK // 4) // CONV_THREADS):
            it, n, c, w, t1, t2 = (p.reg("u32") for _ in range(6))
            p.emit(f"""
                add.u32 {it}, {ctid}, {j * CONV_THREADS}
                and.b32 {n}, {it}, {BNc - 1}
                shr.u32 {c}, {it}, {lg}
                and.b32 {w}, {n}, 31
            """)
            offs = []
            for i in range(4):
                # element (K row 4c+i, column n) of the MN-major tile: block n/32, row
                # 4c+i, 16-byte chunk (n%32)/4 swizzled by the row, word n%4
                o = p.reg("u32")
                p.emit(f"""
                    shr.u32 {t1}, {n}, 5
                    mul.lo.u32 {o}, {t1}, {BK * 128}
                    mad.lo.u32 {o}, {c}, 512, {o}
                    add.u32 {o}, {o}, {i * 128}
                    shr.u32 {t1}, {w}, 2
                    and.b32 {t2}, {c}, 1
                    mad.lo.u32 {t2}, {t2}, 4, {i}
                    xor.b32 {t1}, {t1}, {t2}
                    mad.lo.u32 {o}, {t1}, 16, {o}
                    and.b32 {t2}, {w}, 3
                    mad.lo.u32 {o}, {t2}, 4, {o}
                """)
                offs.append(o)
            rd.append(offs)
            o = p.reg("u32")
            p.emit(f"""
                and.b32 {t1}, {n}, 7
                xor.b32 {t1}, {t1}, {c}
                shl.b32 {t1}, {t1}, 4
                mad.lo.u32 {o}, {n}, 128, {t1}
            """)
            wr.append(o)
    t, s, ph, kb, rph = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {t}, {cta}\nmov.u32 {s}, 0\nmov.u32 {ph}, 0\nmov.u32 {rph}, 0")
    tl, kl = p.label("c_tile"), p.label("c_k")
    pt, ps = p.reg("pred"), p.reg("pred")
    p.place(tl)
    p.emit(f"setp.ge.u32 {pt}, {t}, {ntiles}\n@{pt} bra {finish}\nmov.u32 {kb}, 0")
    p.place(kl)
    fa, ca, base, vb, ra = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {fa}, {s}, 8, {bars}
        add.u32 {ca}, {fa}, {conv0}
        add.u32 {fa}, {fa}, {full0}
        add.u32 {ra}, {bars}, {cread}
    """)
    waits.wait(fa, ph, "convert", finish)
    p.emit(f"mad.lo.u32 {base}, {s}, {stage_bytes}, {ring}\nmad.lo.u32 {vb}, {ctid}, 16, {base}")
    group = 4
    for g0 in range(0, per, group):
        xs = []
        for j in range(g0, min(per, g0 + group)):
            x = [p.reg("b32") for _ in range(4)]
            p.emit(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{vb}+{j * 16 * CONV_THREADS}]")
            xs.append((j, x))
        for j, x in xs:
            parts = _convert(p, cfg, x)
            p.emit(f"st.shared.v4.b32 [{vb}+{j * 16 * CONV_THREADS}], {{{', '.join(h for h, _ in parts)}}}")
            if cfg.split3:
                p.emit(f"st.shared.v4.b32 [{vb}+{j * 16 * CONV_THREADS + raw_bytes}], "
                       f"{{{', '.join(lo for _, lo in parts)}}}")
    if rd:
        bb = p.reg("u32")
        p.emit(f"add.u32 {bb}, {base}, {a_bytes}")
        vals = []
        for offs in rd:
            v = [p.reg("b32") for _ in range(4)]
            for i in range(4):
                ad = p.reg("u32")
                p.emit(f"add.u32 {ad}, {bb}, {offs[i]}\nld.shared.b32 {v[i]}, [{ad}]")
            vals.append(v)
        p.emit(f"mbarrier.arrive.shared::cta.b64 _, [{ra}]")
        waits.wait(ra, rph, "convert", finish)
        p.emit(f"xor.b32 {rph}, {rph}, 1")
        for v, o in zip(vals, wr):
            parts = _convert(p, cfg, v)
            ad = p.reg("u32")
            p.emit(f"add.u32 {ad}, {bb}, {o}")
            p.emit(f"st.shared.v4.b32 [{ad}], {{{', '.join(h for h, _ in parts)}}}")
            if cfg.split3:
                p.emit(f"st.shared.v4.b32 [{ad}+{raw_bytes}], {{{', '.join(lo for _, lo in parts)}}}")
    p.emit(f"""
        fence.proxy.async.shared::cta
        mbarrier.arrive.shared::cta.b64 _, [{ca}]
        add.u32 {s}, {s}, 1
        setp.eq.u32 {ps}, {s}, {cfg.stages}
        @{ps} mov.u32 {s}, 0
        @{ps} xor.b32 {ph}, {ph}, 1
        add.u32 {kb}, {kb}, 1
        setp.lt.u32 {ps}, {kb}, {kblocks}
        @{ps} bra {kl}
        add.u32 {t}, {t}, {nct}
        bra {tl}
    """)


def _emit_direct_loader(p: Ptx, cfg: GemmConfig, ptr: dict, tid, ring, bars, empty0, conv0, a_bytes,
                        raw_bytes, stage_bytes, kblocks, cta, nct, ntiles, waits: Waits, finish: str, ks: int = 1) -> None:
    """Converter warps that fetch the operands from global memory themselves (no TMA): for
    rows that are not 16-byte aligned (emmy's odd-shaped fixtures), 16-bit sources (widened
    exactly) and mixed operand types.  Per stage each of the 128 threads loads its
    elements of the 128 x 32 A tile and the BN x 32 B tile (out-of-range rows, columns and
    K zero-filled: the loads are predicated), converts them like ``_emit_split_tf32`` and
    writes them into the K-major 128-byte-swizzled layout the MMAs read.  The stage is
    taken once the MMAs released it (empty[stage]) and handed over on conv[stage]."""
    M, N, K, BN = cfg.M, cfg.N, cfg.K, cfg.BN
    ea, eb = ELEM_BYTES[cfg.a_dtype], ELEM_BYTES[cfg.b_dtype]
    ctid, lane, grp, l4, lw, t1 = (p.reg("u32") for _ in range(6))
    p.emit(f"""
        sub.u32 {ctid}, {tid}, {GEMM_THREADS}
        and.b32 {lane}, {ctid}, 31
        shr.u32 {grp}, {ctid}, 5
        shr.u32 {l4}, {lane}, 2
        and.b32 {lw}, {lane}, 3
        shl.b32 {lw}, {lw}, 2
    """)
    # K-major rows grp + 4j: row & 7 = grp + 4 (j & 1), so two chunk offsets serve all j
    kmaj = []
    for par in (0, 1):
        o = p.reg("u32")
        p.emit(f"""
            add.u32 {t1}, {grp}, {4 * par}
            xor.b32 {t1}, {t1}, {l4}
            shl.b32 {t1}, {t1}, 4
            mad.lo.u32 {o}, {grp}, 128, {t1}
            add.u32 {o}, {o}, {lw}
        """)
        kmaj.append(o)
    # MN-major B columns lane + 32c, K rows grp + 4q: chunk q ^ (lane & 7), word grp
    mnq = []
    if not cfg.b_kmajor:
        l7, gw = p.reg("u32"), p.reg("u32")
        p.emit(f"and.b32 {l7}, {lane}, 7\nshl.b32 {gw}, {grp}, 2")
        for q in range(8):
            o = p.reg("u32")
            p.emit(f"""
                xor.b32 {t1}, {l7}, {q}
                shl.b32 {t1}, {t1}, 4
                mad.lo.u32 {o}, {lane}, 128, {t1}
                add.u32 {o}, {o}, {gw}
            """)
            mnq.append(o)
    nbb = BN // 32
    t, s, ph, kb = (p.reg("u32") for _ in range(4))
    p.emit(f"mov.u32 {t}, {cta}\nmov.u32 {s}, 0\nmov.u32 {ph}, 0")
    tl, kl = p.label("d_tile"), p.label("d_k")
    pt, ps = p.reg("pred"), p.reg("pred")
    p.place(tl)
    p.emit(f"setp.ge.u32 {pt}, {t}, {ntiles}\n@{pt} bra {finish}\nmov.u32 {kb}, 0")
    bt, mt, nt = _tile_coords(p, cfg, t, ks)
    m0, n0, kb0 = p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"mul.lo.u32 {m0}, {mt}, {cfg.MT}\nmul.lo.u32 {n0}, {nt}, {BN}\n"
           f"rem.u32 {kb0}, {t}, {ks}\nmul.lo.u32 {kb0}, {kb0}, {kblocks}")
    p.place(kl)
    ea_, ca, par, base, k0 = (p.reg("u32") for _ in range(5))
    p.emit(f"""
        mad.lo.u32 {ea_}, {s}, 8, {bars}
        add.u32 {ca}, {ea_}, {conv0}
        add.u32 {ea_}, {ea_}, {empty0}
        xor.b32 {par}, {ph}, 1
        add.u32 {k0}, {kb}, {kb0}
        mul.lo.u32 {k0}, {k0}, 32
    """)
    waits.wait(ea_, par, "convert", finish)
    p.emit(f"mad.lo.u32 {base}, {s}, {stage_bytes}, {ring}")

    def load(dtype, adr, off, pred):
        v = p.reg("b32")
        p.emit(f"mov.b32 {v}, 0")
        if dtype == "f64":        # an f64 operand whose products the IR takes in f32
            d = p.reg("f64")
            p.emit(f"mov.f64 {d}, 0d0000000000000000\n@{pred} ld.global.f64 {d}, [{adr}+{off}]\n"
                   f"cvt.rn.f32.f64 {v}, {d}")
        elif dtype == "f32":
            p.emit(f"@{pred} ld.global.b32 {v}, [{adr}+{off}]")
        else:
            h = p.reg("b16")
            up = "cvt.f32.f16" if dtype == "f16" else "cvt.f32.bf16"
            p.emit(f"mov.b16 {h}, 0\n@{pred} ld.global.b16 {h}, [{adr}+{off}]\n{up} {v}, {h}")
        return v

    def store(items):
        for x, off in items:
            (hi, lo), = _convert(p, cfg, [x])
            ad = p.reg("u32")
            p.emit(f"add.u32 {ad}, {base}, {off[0]}")
            p.emit(f"st.shared.b32 [{ad}+{off[1]}], {hi}")
            if cfg.split3:
                p.emit(f"st.shared.b32 [{ad}+{off[1] + raw_bytes}], {lo}")

    def limit(x):
        if x >= 2 ** 31:
            raise NotImplementedError("operand offsets beyond 32 bits")
        return x

    # A [batch, M, K]: rows m0 + grp + 4j, K k0 + lane
    ra, kk, pk = p.reg("u32"), p.reg("u32"), p.reg("pred")
    aad, w = p.reg("b64"), p.reg("b64")
    p.emit(f"""
        add.u32 {ra}, {m0}, {grp}
        add.u32 {kk}, {k0}, {lane}
        setp.lt.u32 {pk}, {kk}, {K}
        mad.lo.u32 {t1}, {bt}, {M}, {ra}
        mul.wide.u32 {aad}, {t1}, {K}
        cvt.u64.u32 {w}, {kk}
        add.s64 {aad}, {aad}, {w}
        mad.lo.s64 {aad}, {aad}, {ea}, {ptr[cfg.a_param]}
    """)
    for g0 in range(0, 32, 8):
        items = []
        for j in range(g0, g0 + 8):
            pj = p.reg("pred")
            if M - 4 * j <= 0:
                continue
            p.emit(f"setp.lt.and.u32 {pj}, {ra}, {M - 4 * j}, {pk}")
            items.append((load(cfg.a_dtype, aad, limit(j * 4 * K * ea), pj), (kmaj[j & 1], j * 512)))
        store(items)
    bad, rb = p.reg("b64"), p.reg("u32")
    if cfg.b_kmajor:
        # B [batch, N, K]: rows n0 + grp + 4i, K k0 + lane
        p.emit(f"""
            add.u32 {rb}, {n0}, {grp}
            mad.lo.u32 {t1}, {bt}, {N}, {rb}
            mul.wide.u32 {bad}, {t1}, {K}
            cvt.u64.u32 {w}, {kk}
            add.s64 {bad}, {bad}, {w}
            mad.lo.s64 {bad}, {bad}, {eb}, {ptr[cfg.b_param]}
        """)
        for g0 in range(0, BN // 4, 8):
            items = []
            for i in range(g0, min(BN // 4, g0 + 8)):
                pi = p.reg("pred")
                if N - 4 * i <= 0:
                    continue
                p.emit(f"setp.lt.and.u32 {pi}, {rb}, {N - 4 * i}, {pk}")
                items.append((load(cfg.b_dtype, bad, limit(i * 4 * K * eb), pi), (kmaj[i & 1], a_bytes + i * 512)))
            store(items)
    else:
        # B [batch, K, N]: K rows k0 + grp + 4q, columns n0 + lane + 32c
        kb_, cn = p.reg("u32"), p.reg("u32")
        p.emit(f"""
            add.u32 {kb_}, {k0}, {grp}
            add.u32 {cn}, {n0}, {lane}
            mad.lo.u32 {t1}, {bt}, {K}, {kb_}
            mul.wide.u32 {bad}, {t1}, {N}
            cvt.u64.u32 {w}, {cn}
            add.s64 {bad}, {bad}, {w}
            mad.lo.s64 {bad}, {bad}, {eb}, {ptr[cfg.b_param]}
        """)
        pq = [p.reg("pred") for _ in range(8)]
        pc = [p.reg("pred") for _ in range(nbb)]
        for q in range(8):
            p.emit(f"setp.lt.u32 {pq[q]}, {kb_}, {K - 4 * q}" if K - 4 * q > 0 else f"setp.ne.u32 {pq[q]}, 0, 0")
        for c in range(nbb):
            p.emit(f"setp.lt.u32 {pc[c]}, {cn}, {N - 32 * c}" if N - 32 * c > 0 else f"setp.ne.u32 {pc[c]}, 0, 0")
        for q in range(8):
            items = []
            for c in range(nbb):
                pi = p.reg("pred")
                p.emit(f"and.pred {pi}, {pq[q]}, {pc[c]}")
                items.append((load(cfg.b_dtype, bad, limit((4 * q * N + 32 * c) * eb), pi),
                              (mnq[q], a_bytes + c * 4096)))
            store(items)
    p.emit(f"""
        fence.proxy.async.shared::cta
        mbarrier.arrive.shared::cta.b64 _, [{ca}]
        add.u32 {s}, {s}, 1
        setp.eq.u32 {ps}, {s}, {cfg.stages}
        @{ps} mov.u32 {s}, 0
        @{ps} xor.b32 {ph}, {ph}, 1
        add.u32 {kb}, {kb}, 1
        setp.lt.u32 {ps}, {kb}, {kblocks}
        @{ps} bra {kl}
        add.u32 {t}, {t}, {nct}
        bra {tl}
    """)


def _emit_epilogue(p: Ptx, cfg: GemmConfig, ptr: dict, bars, tfull0, tempty0, tbase, warp, lane,
                   cta, nct, ntiles, waits: Waits, finish: str, crank=None, ltempty=None,
                   ks: int = 1, tail=None, epi_stage=None) -> None:
    """TMEM accumulator -> fused epilogue ops -> C, one thread per row.  With ``ks`` K slices
    per tile, each unit first writes its f32 partial to a workspace; per warp quarter of the
    tile a ticket counts the slices in, and the warp that takes the last one sums the
    slices in slice order (deterministic), applies the epilogue and writes C."""
    M, N, BM, BN = cfg.M, cfg.N, cfg.BM, cfg.BN
    cb = ELEM_BYTES[cfg.c]
    q, row_t = p.reg("u32"), p.reg("u32")
    p.emit(f"and.b32 {q}, {warp}, 3\nmad.lo.u32 {row_t}, {q}, 32, {lane}")
    wbuf = rsub = csub = None
    if epi_stage is not None:
        # this warp's staging rows, and the (row, 16-byte column piece) each lane stores
        ring_r, epi_off = epi_stage
        wbuf, rsub, csub = p.reg("u32"), p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {wbuf}, {q}, {32 * EPI_ROW}, {ring_r}\nadd.u32 {wbuf}, {wbuf}, {epi_off}\n"
               f"shr.u32 {rsub}, {lane}, 2\nand.b32 {csub}, {lane}, 3")
    lane_off = p.reg("u32")
    p.emit(f"shl.b32 {lane_off}, {q}, 21")           # (q * 32) << 16: the warp's TMEM lane quarter
    cptr = ptr[cfg.c_param]
    extra, kinds = {}, {}
    for op in cfg.epilogue:
        if op[0] in ("bias", "residual"):
            extra[op[1]] = ptr[op[1]]
            kinds[op[1]] = op[0]
        elif op[0] == "lambda":
            for _, kind, buf in op[2]:
                extra[buf] = ptr[buf]
                kinds[buf] = kind
    scale = None
    for op in cfg.epilogue:
        if op[0] == "scale2":
            sa, sb, scale = p.reg("f32"), p.reg("f32"), p.reg("f32")
            p.emit(f"ld.global.f32 {sa}, [{ptr[op[1]]}]\nld.global.f32 {sb}, [{ptr[op[2]]}]\n"
                   f"mul.rn.f32 {scale}, {sa}, {sb}")
    t, tc = p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {t}, {cta}\nmov.u32 {tc}, 0")
    el, ed = p.label("e_tile"), p.label("e_done")
    p.place(el)
    pt = p.reg("pred")
    p.emit(f"setp.ge.u32 {pt}, {t}, {ntiles}\n@{pt} bra {ed}")
    ab, aph, tfa, tea = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        rem.u32 {ab}, {tc}, {cfg.acc_bufs}
        div.u32 {aph}, {tc}, {cfg.acc_bufs}
        and.b32 {aph}, {aph}, 1
        mad.lo.u32 {tfa}, {ab}, 8, {bars}
        add.u32 {tea}, {tfa}, {tempty0}
        add.u32 {tfa}, {tfa}, {tfull0}
    """)
    waits.wait(tfa, aph, "epilogue", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    if tail is None:
        bt, mt, nt = _tile_coords(p, cfg, t, ks)
        psl = v = None
    else:
        bt, mt, nt, _, _, psl, v = _unit_plan(p, cfg, t, 1, 0, tail)
    row, n0, taddr = p.reg("u32"), p.reg("u32"), p.reg("u32")
    prow = p.reg("pred")
    if crank is not None:   # the CTA's 128 rows of the pair's 256-row tile
        rt2 = p.reg("u32")
        p.emit(f"mad.lo.u32 {rt2}, {crank}, {BM}, {row_t}")
    else:
        rt2 = row_t
    p.emit(f"""
        mad.lo.u32 {row}, {mt}, {cfg.MT}, {rt2}
        mul.lo.u32 {n0}, {nt}, {BN}
        setp.lt.u32 {prow}, {row}, {M}
        mad.lo.u32 {taddr}, {ab}, {BN}, {tbase}
        add.u32 {taddr}, {taddr}, {lane_off}
    """)
    # element offset of (batch, row, n0) in C
    off, cadr = p.reg("b64"), p.reg("b64")
    wide = p.reg("b64")
    p.emit(f"""
        mul.wide.u32 {off}, {bt}, {M}
        cvt.u64.u32 {wide}, {row}
        add.s64 {off}, {off}, {wide}
        mul.lo.s64 {off}, {off}, {N}
        cvt.u64.u32 {wide}, {n0}
        add.s64 {off}, {off}, {wide}
        mad.lo.s64 {cadr}, {off}, {cb}, {cptr}
    """)
    res_adr = {}
    for name, bp in extra.items():
        a = p.reg("b64")
        kind = kinds[name]
        esz = ELEM_BYTES[_elem_dtype(cfg, name)]
        if kind == "residual":
            p.emit(f"mad.lo.s64 {a}, {off}, {esz}, {bp}")
        else:   # bias over N: element n0
            w2 = p.reg("b64")
            p.emit(f"cvt.u64.u32 {w2}, {n0}\nmad.lo.s64 {a}, {w2}, {esz}, {bp}")
        res_adr[name] = a
    nchunks = BN // 32
    regs = [p.reg("b32") for _ in range(32)]
    if wbuf is not None:
        # the warp's first row (the lane's row minus its lane) and the address of
        # (row rsub, piece csub) of its chunk 0: lane l stores rows l / 4 + 8 i
        rowq0, sadr, w64 = p.reg("u32"), p.reg("b64"), p.reg("b64")
        p.emit(f"""
            sub.u32 {rowq0}, {row}, {lane}
            mul.wide.u32 {w64}, {lane}, {N * cb}
            sub.s64 {sadr}, {cadr}, {w64}
            mul.wide.u32 {w64}, {rsub}, {N * cb}
            add.s64 {sadr}, {sadr}, {w64}
            mul.wide.u32 {w64}, {csub}, 16
            add.s64 {sadr}, {sadr}, {w64}
        """)
    if cfg.zero_slots and cfg.c != "f32":
        raise NotImplementedError("split-K partial slices other than f32")
    def load_chunk(ch):
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{taddr}+{ch * 32}]")
        p.emit("tcgen05.wait::ld.sync.aligned")
        if ch == nchunks - 1:
            # the accumulator is in registers: hand the buffer back to the MMA warp
            if ltempty is not None:   # the leader CTA issues the MMAs: release to its barrier
                ra = p.reg("u32")
                p.emit(f"tcgen05.fence::before_thread_sync\nmad.lo.u32 {ra}, {ab}, 8, {ltempty}\n"
                       f"mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{ra}]")
            else:
                p.emit(f"tcgen05.fence::before_thread_sync\nmbarrier.arrive.shared::cta.b64 _, [{tea}]")

    def store_chunk_staged(ch, vals):
        """Each lane's row of 32 results into the warp's staging rows, then the warp
        stores 8 rows x 64 contiguous bytes per instruction (4 instructions a chunk)."""
        cvt = "cvt.rn.bf16x2.f32" if cfg.c == "bf16" else "cvt.rn.f16x2.f32"
        packed = [p.reg("b32") for _ in range(16)]
        for i in range(16):
            p.emit(f"{cvt} {packed[i]}, {vals[2 * i + 1]}, {vals[2 * i]}")
        wrow = p.reg("u32")
        p.emit(f"mad.lo.u32 {wrow}, {lane}, {EPI_ROW}, {wbuf}")
        for g in range(4):
            p.emit(f"st.shared.v4.b32 [{wrow}+{16 * g}], {{{', '.join(packed[4 * g:4 * g + 4])}}}")
        p.emit("bar.warp.sync -1")
        rd, colr, grow = p.reg("u32"), p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {rd}, {rsub}, {EPI_ROW}, {wbuf}\nmad.lo.u32 {rd}, {csub}, 16, {rd}\n"
               f"mad.lo.u32 {colr}, {csub}, 8, {n0}\nadd.u32 {colr}, {colr}, {ch * 32}")
        pc = p.reg("pred")
        p.emit(f"setp.lt.u32 {pc}, {colr}, {N}")
        for i in range(4):
            x = [p.reg("b32") for _ in range(4)]
            pg = p.reg("pred")
            p.emit(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{rd}+{8 * i * EPI_ROW}]\n"
                   f"add.u32 {grow}, {rowq0}, {rsub}\nadd.u32 {grow}, {grow}, {8 * i}\n"
                   f"setp.lt.and.u32 {pg}, {grow}, {M}, {pc}\n"
                   f"@{pg} st.global.v4.b32 [{sadr}+{8 * i * N * cb + ch * 64}], {{{', '.join(x)}}}")
        p.emit("bar.warp.sync -1")

    def store_chunk(ch, vals):
        vals = _apply_epilogue(p, cfg, vals, scale, res_adr, ch, prow, n0)
        if wbuf is not None:
            store_chunk_staged(ch, vals)
            return
        skip = p.label("st_skip")
        col0 = ch * 32
        p.emit(f"@!{prow} bra {skip}")
        if cfg.c in ("bf16", "f16") and N % 8 == 0:
            cvt = "cvt.rn.bf16x2.f32" if cfg.c == "bf16" else "cvt.rn.f16x2.f32"
            packed = [p.reg("b32") for _ in range(16)]
            for i in range(16):
                # the first element of a pair goes to the low half (lower address)
                p.emit(f"{cvt} {packed[i]}, {vals[2 * i + 1]}, {vals[2 * i]}")
            for g in range(4):
                pg = p.reg("pred")
                colr = p.reg("u32")
                p.emit(f"add.u32 {colr}, {n0}, {col0 + 8 * g}\nsetp.lt.u32 {pg}, {colr}, {N}")
                p.emit(f"@{pg} st.global.v4.b32 [{cadr}+{(col0 + 8 * g) * 2}], "
                       f"{{{', '.join(packed[4 * g:4 * g + 4])}}}")
        elif cfg.c == "f32" and N % 4 == 0:
            for g in range(8):
                pg, colr = p.reg("pred"), p.reg("u32")
                p.emit(f"add.u32 {colr}, {n0}, {col0 + 4 * g}\nsetp.lt.u32 {pg}, {colr}, {N}")
                p.emit(f"@{pg} st.global.v4.f32 [{cadr}+{(col0 + 4 * g) * 4}], "
                       f"{{{', '.join(vals[4 * g:4 * g + 4])}}}")
        elif cfg.c == "f64":
            if cfg.zero_slots:
                raise NotImplementedError("split-K partial slices other than f32")
            for i in range(32):
                pg, colr, d = p.reg("pred"), p.reg("u32"), p.reg("f64")
                p.emit(f"add.u32 {colr}, {n0}, {col0 + i}\nsetp.lt.u32 {pg}, {colr}, {N}\n"
                       f"cvt.f64.f32 {d}, {vals[i]}\n@{pg} st.global.f64 [{cadr}+{(col0 + i) * 8}], {d}")
        else:
            for i in range(32):
                pg, colr = p.reg("pred"), p.reg("u32")
                p.emit(f"add.u32 {colr}, {n0}, {col0 + i}\nsetp.lt.u32 {pg}, {colr}, {N}")
                if cfg.c == "f32":
                    p.emit(f"@{pg} st.global.f32 [{cadr}+{(col0 + i) * 4}], {vals[i]}")
                else:
                    h = p.reg("b16")
                    cvt = "cvt.rn.bf16.f32" if cfg.c == "bf16" else "cvt.rn.f16.f32"
                    p.emit(f"{cvt} {h}, {vals[i]}\n@{pg} st.global.b16 [{cadr}+{(col0 + i) * 2}], {h}")
        p.place(skip)

    if ks > 1:
        l_next = _emit_ksplit_partial(p, cfg, ks, t, row_t, lane, q, regs, nchunks, load_chunk)
        for ch in range(nchunks):
            store_chunk(ch, _ksplit_sum(p, cfg, ks, t, row_t, ch))
    elif tail is not None:
        # whole tiles store straight from TMEM; sliced tail units go through the workspace
        l_sl, l_join = p.label("e_sliced"), p.label("e_join")
        p.emit(f"@{psl} bra {l_sl}")
        for ch in range(nchunks):
            load_chunk(ch)
            vals = [p.reg("f32") for _ in range(32)]
            for i in range(32):
                p.emit(f"mov.b32 {vals[i]}, {regs[i]}")
            store_chunk(ch, vals)
        p.emit(f"bra {l_join}")
        p.place(l_sl)
        ts = tail[1]
        l_next = _emit_ksplit_partial(p, cfg, ts, v, rt2, lane, q, regs, nchunks, load_chunk, crank)
        for ch in range(nchunks):
            store_chunk(ch, _ksplit_sum(p, cfg, ts, v, rt2, ch))
        p.place(l_join)
    else:
        l_next = None
        for ch in range(nchunks):
            load_chunk(ch)
            vals = [p.reg("f32") for _ in range(32)]
            for i in range(32):
                p.emit(f"mov.b32 {vals[i]}, {regs[i]}")
            store_chunk(ch, vals)
    if l_next is not None:
        p.place(l_next)
    p.emit(f"""
        add.u32 {tc}, {tc}, 1
        add.u32 {t}, {t}, {nct}
        bra {el}
    """)
    p.place(ed)
    p.emit(f"bra {finish}")


def _emit_ksplit_partial(p: Ptx, cfg: GemmConfig, ks: int, t: str, row_t: str, lane: str,
                         q: str, regs: list, nchunks: int, load_chunk, crank=None) -> str:
    """Write this unit's accumulator rows to the workspace and take the warp quarter's
    ticket; returns the label the warps that are not last jump to (the next unit)."""
    BN, MT = cfg.BN, cfg.MT
    ws, tk = p.reg("b64"), p.reg("b64")
    p.emit(f"ld.param.u64 {ws}, [param__ksplit_ws]\ncvta.to.global.u64 {ws}, {ws}\n"
           f"ld.param.u64 {tk}, [param__ksplit_tickets]\ncvta.to.global.u64 {tk}, {tk}")
    # the workspace holds one f32 partial per unit, [unit][column / 4][row][4]: the lanes
    # (consecutive rows) of a warp store consecutive 16-byte pieces, 512 bytes per warp
    # store, and the slices are summed with the same coalesced loads
    wrow = _ws_row(p, ws, t, row_t, MT, BN)
    for ch in range(nchunks):
        load_chunk(ch)
        for g in range(8):
            p.emit(f"st.global.v4.b32 [{wrow}+{(ch * 8 + g) * MT * 16}], {{{', '.join(regs[4 * g:4 * g + 4])}}}")
    # every lane's stores before lane 0's ticket; the ticket of (tile, warp quarter).  Lane
    # 0 takes it with an acq_rel atom; the warp barrier after the broadcast orders the
    # other lanes' later reads of the other slices after that acquire (then each lane's
    # own fence)
    tile, ta, old, last = p.reg("u32"), p.reg("b64"), p.reg("u32"), p.reg("u32")
    p0, pl = p.reg("pred"), p.reg("pred")
    l_next = p.label("ks_next")
    p.emit(f"""
        fence.acq_rel.gpu
        bar.warp.sync -1
        div.u32 {tile}, {t}, {ks}
        {f"mad.lo.u32 {tile}, {tile}, 2, {crank}" if crank is not None else ""}
        mad.lo.u32 {tile}, {tile}, 4, {q}
        mul.wide.u32 {ta}, {tile}, 4
        add.s64 {ta}, {ta}, {tk}
        setp.eq.u32 {p0}, {lane}, 0
        mov.u32 {last}, 0
        @{p0} atom.acq_rel.gpu.global.add.u32 {old}, [{ta}], 1
        @{p0} setp.eq.u32 {pl}, {old}, {ks - 1}
        @{p0} selp.u32 {last}, 1, 0, {pl}
        shfl.sync.idx.b32 {last}, {last}, 0, 31, -1
        bar.warp.sync -1
        setp.eq.u32 {pl}, {last}, 0
        @{pl} bra {l_next}
        @{p0} st.relaxed.gpu.global.u32 [{ta}], 0
        fence.acq_rel.gpu
    """)
    return l_next


def _ws_row(p: Ptx, ws: str, unit: str, row: str, MT: int, BN: int) -> str:
    """Address of (unit, first column group, row) in the [unit][column / 4][row][4] f32
    workspace; column group g of chunk ch is (ch * 8 + g) * MT * 16 bytes further."""
    a, r = p.reg("b64"), p.reg("b64")
    p.emit(f"mul.wide.u32 {a}, {unit}, {MT * BN * 4}\nadd.s64 {a}, {a}, {ws}\n"
           f"mul.wide.u32 {r}, {row}, 16\nadd.s64 {a}, {a}, {r}")
    return a


def _ksplit_sum(p: Ptx, cfg: GemmConfig, ks: int, t: str, row_t: str, ch: int) -> list:
    """Columns 32 ch .. 32 ch + 31 of the thread's row summed over the tile's slices in
    slice order (L2 loads: the other slices were written by other CTAs)."""
    BN, MT = cfg.BN, cfg.MT
    ws = p.reg("b64")
    p.emit(f"ld.param.u64 {ws}, [param__ksplit_ws]\ncvta.to.global.u64 {ws}, {ws}")
    u0, w = p.reg("u32"), p.reg("u32")
    # unit of slice 0 of this tile: t - t % ks
    p.emit(f"rem.u32 {u0}, {t}, {ks}\nsub.u32 {u0}, {t}, {u0}")
    acc = [p.reg("f32") for _ in range(32)]
    # the loads of up to four slices are in flight together (their own registers), then
    # added in slice order: one L2 round trip per group of slices, the same sum
    for g0 in range(0, ks, 4):
        group = list(range(g0, min(ks, g0 + 4)))
        bufs = {sl: (acc if sl == 0 else [p.reg("f32") for _ in range(32)]) for sl in group}
        for sl in group:
            p.emit(f"add.u32 {w}, {u0}, {sl}")
            a = _ws_row(p, ws, w, row_t, MT, BN)
            dst = bufs[sl]
            for g in range(8):
                p.emit(f"ld.global.cg.v4.f32 {{{', '.join(dst[4 * g:4 * g + 4])}}}, "
                       f"[{a}+{(ch * 8 + g) * MT * 16}]")
        for sl in group:
            if sl:
                for i in range(32):
                    p.emit(f"add.rn.f32 {acc[i]}, {acc[i]}, {bufs[sl][i]}")
    return acc


def _load_operand(p: Ptx, cfg: GemmConfig, buf: str, adr: str, ch: int, i: int, prow, n0) -> str:
    """Element (row, n0 + 32 ch + i) of an epilogue operand as f32; 0 outside C."""
    dt = _elem_dtype(cfg, buf)
    pin, col, r = p.reg("pred"), p.reg("u32"), p.reg("f32")
    p.emit(f"add.u32 {col}, {n0}, {ch * 32 + i}\nsetp.lt.and.u32 {pin}, {col}, {cfg.N}, {prow}\n"
           f"mov.f32 {r}, 0f00000000")
    if dt == "f32":
        p.emit(f"@{pin} ld.global.f32 {r}, [{adr}+{(ch * 32 + i) * 4}]")
    else:
        h = p.reg("b16")
        up = "cvt.f32.f16" if dt == "f16" else "cvt.f32.bf16"
        p.emit(f"mov.b16 {h}, 0\n@{pin} ld.global.b16 {h}, [{adr}+{(ch * 32 + i) * 2}]\n{up} {r}, {h}")
    return r


def _apply_epilogue(p: Ptx, cfg: GemmConfig, vals: list, scale, res_adr: dict, ch: int,
                    prow, n0) -> list:
    """Fused elementwise ops on one 32-column chunk of a row (f32 registers)."""
    for op in cfg.epilogue:
        kind = op[0]
        if kind == "scale2":
            for v in vals:
                p.emit(f"mul.rn.f32 {v}, {v}, {scale}")
        elif kind == "relu":
            for v in vals:
                p.emit(f"max.f32 {v}, {v}, 0f00000000")
        elif kind == "round":
            rdt = op[1] if len(op) > 1 else cfg.c
            rdown = "cvt.rn.f16.f32" if rdt == "f16" else "cvt.rn.bf16.f32"
            rup = "cvt.f32.f16" if rdt == "f16" else "cvt.f32.bf16"
            for v in vals:
                h = p.reg("b16")
                p.emit(f"{rdown} {h}, {v}\n{rup} {v}, {h}")
        elif kind in ("bias", "residual"):
            for i, v in enumerate(vals):
                r = _load_operand(p, cfg, op[1], res_adr[op[1]], ch, i, prow, n0)
                p.emit(f"add.rn.f32 {v}, {v}, {r}")
        elif kind == "lambda":
            from ..stmts import ScalarCtx, Val, lower_body
            lam, operands, consts = op[1], op[2], dict(op[3])
            for i, v in enumerate(vals):
                ctx = ScalarCtx(p, constants=consts, half_results=True)
                ctx.env[lam.params[0]] = Val(v, "f32")
                for lname, _, buf in operands:
                    ctx.env[lname] = Val(_load_operand(p, cfg, buf, res_adr[buf], ch, i, prow, n0), "f32")
                lower_body(ctx, lam.body)
                p.emit(f"mov.f32 {v}, {ctx.f32(lam.results[0])}")
        else:
            raise NotImplementedError(f"GEMM epilogue {kind}")
    return vals


def _elem_dtype(cfg: GemmConfig, buf: str) -> str:
    """A 16-bit epilogue operand's dtype (the IR's; the C type when not recorded)."""
    return dict(cfg.operand_dtypes).get(buf, cfg.c)


# ---------------------------------------------------------------------------
# recognising the IR's matmul family


def _walk(body):
    for s in body:
        yield s
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple):
                yield from _walk(sub)


def _vars(expr) -> set:
    from ..stmts import expr_vars
    return expr_vars(expr)


def analyze(spec) -> GemmConfig:
    """Identify A, B (and its major order), C and the epilogue of a matmul kernel."""
    stmts = list(_walk(spec.body))
    kinds = {type(s).__name__ for s in stmts}
    if "MmaSyncPtx" not in kinds or "FragmentRowReduce" in kinds:
        raise NotImplementedError("not a tensor-core matmul")
    stores = [s for s in stmts if type(s).__name__ == "RegStore"]
    if not stores or len({s.dst_buffer for s in stores}) != 1:
        raise NotImplementedError("matmul without a single RegStore output")
    if any(getattr(s, "extra_frags", None) for s in stores):
        raise NotImplementedError("a store combining several accumulators (two matmuls)")
    cname = stores[0].dst_buffer
    # emmy's split-K with atomic partial sums into the zeroed C (``x_h_attn_odd``): the whole
    # K in one pass gives the same sum
    atomic = any(s.atomic for s in stores)
    if atomic and cname not in spec.zero_outputs:
        raise NotImplementedError("split-K partial matmul (atomic RegStore) into a C that is not zeroed")
    # emmy's split-K schedule: a `*_ks` tile axis gives each CTA one K slice and the
    # partial products go to slice ks of an f32 [S, ..., M, N] buffer that a second
    # kernel sums; here the whole K runs in one pass into slice 0, the others are zeroed
    tile = spec.body[0] if len(spec.body) == 1 and type(spec.body[0]).__name__ == "Tile" else None
    ks_axes = [a for a in (tile.axes if tile else ()) if a.name.endswith("_ks")]
    if len(ks_axes) > 1:
        raise NotImplementedError("more than one split-K axis")
    ks = ks_axes[0] if ks_axes else None
    # the K loop: the Loop that (transitively) holds the MmaSyncPtx statements
    kvar = None
    for s in stmts:
        if type(s).__name__ in ("Loop", "StridedLoop") and any(
                type(x).__name__ == "MmaSyncPtx" for x in _walk(s.body)):
            kvar = s.axis.name
            break
    # operand sources: smem staging (CpAsyncCopy / Write of loaded values) or gmem-direct
    smem_src, smem_cast = {}, {}
    defs = {}
    for s in stmts:
        k = type(s).__name__
        if k == "Load":
            for n in s.names:
                defs[n] = s
        elif k == "Assign":
            defs[s.name] = s
    for s in stmts:
        k = type(s).__name__
        if k == "CpAsyncCopy":
            smem_src[s.smem] = (s.src, s.src_index)
        elif k == "Write" and s.output not in spec.buffers and s.values:
            # a shared tile written from loaded values, possibly cast (``x.to(bf16)``)
            d, cast = defs.get(s.values[0]), None
            while d is not None and type(d).__name__ == "Assign" and d.op.name == "copy":
                dt = getattr(d.dtype, "name", None)
                cast = dt if dt in ("bf16", "f16") else cast
                d = defs.get(d.args[0])
            if d is not None and type(d).__name__ == "Load" and d.input in spec.buffers:
                smem_src[s.output] = (d.input, d.index)
                smem_cast[s.output] = cast
    role_src, role_cast = {}, {}
    for s in stmts:
        if type(s).__name__ == "LdmatrixLoad":
            buf = s.src_buffer
            src = smem_src.get(buf, (buf, s.src_index) if buf in spec.buffers else None)
            if src is None:
                raise NotImplementedError(f"cannot trace operand {s.frag} to a buffer")
            role_src.setdefault(s.role, src)
            role_cast.setdefault(s.role, smem_cast.get(buf))
    if set(role_src) != {"a", "b"}:
        raise NotImplementedError("matmul operands not found")
    (aname, aidx), (bname, bidx) = role_src["a"], role_src["b"]
    A, B, C = spec.param(aname), spec.param(bname), spec.param(cname)
    # f32 operands cast to a 16-bit type on the way into shared memory: the tf32 template
    # with the same rounding (the 16-bit products are exact either way)
    f32_cast = A.dtype == B.dtype == "f32" and role_cast["a"] == role_cast["b"] and \
        role_cast["a"] in ("bf16", "f16")
    if not f32_cast and (A.dtype != B.dtype or A.dtype not in ("f16", "bf16")):
        raise NotImplementedError(f"matmul operands {A.dtype}/{B.dtype}: TMA feeds 16-bit operands")
    if C.dtype not in ("f16", "bf16", "f32"):
        raise NotImplementedError(f"matmul output {C.dtype}")
    if kvar is None:
        raise NotImplementedError("no K loop")

    def k_dim(index) -> int:
        dims = [i for i, e in enumerate(index) if kvar in _vars(e)]
        if len(dims) != 1:
            raise NotImplementedError("K axis not identifiable in an operand index")
        return dims[0]
    if k_dim(aidx) != len(A.shape) - 1:
        raise NotImplementedError("A operand is not K-major")
    b_kmajor = k_dim(bidx) == len(B.shape) - 1
    M, K = A.shape[-2], A.shape[-1]
    N = B.shape[-2] if b_kmajor else B.shape[-1]
    if (B.shape[-1] if b_kmajor else B.shape[-2]) != K or tuple(C.shape[-2:]) != (M, N):
        raise NotImplementedError("operand shapes do not form a matmul")
    split = {}
    cdims = C.shape
    if ks is not None and not atomic:
        S = int(ks.extent.value)
        kloop = next(x for x in stmts if type(x).__name__ in ("Loop", "StridedLoop") and x.axis.name == kvar)
        first = stores[0].dst_index[0] if stores[0].dst_index else None
        if C.dtype != "f32" or cdims[0] != S or _vars(first) != {ks.name} or \
                S * int(kloop.axis.extent.value) != K:
            raise NotImplementedError("split-K partial that does not slice K exactly")
        cdims = cdims[1:]
        split = dict(zero_slots=S - 1, slot_stride=int(math.prod(cdims)))
    batch = int(math.prod(cdims[:-2])) if len(cdims) > 2 else 1
    if batch > 1 and (math.prod(A.shape[:-2]) != batch or math.prod(B.shape[:-2]) != batch):
        raise NotImplementedError("broadcast batch operands")
    eb = 4 if f32_cast else 2
    aligned = not ((K * eb) % 16 or (not b_kmajor and (N * eb) % 16))
    epi = _epilogue_ops(spec, stores[0])
    if atomic and epi:
        raise NotImplementedError("an epilogue on atomic partial sums")
    if f32_cast or not aligned:
        # the tf32 template: f32 operands rounded as the IR casts them, or 16-bit operands
        # (exact in tf32) fetched by the converter warps where TMA cannot address the rows
        if f32_cast and C.dtype != "f32":
            raise NotImplementedError("cast-operand matmul with a 16-bit output")
        od = tuple((q.name, q.dtype) for q in spec.params)
        return GemmConfig(M=M, N=N, K=K, batch=batch, ab="f32", c=C.dtype, b_kmajor=b_kmajor,
                          **choose_tiling_f32(M, N, batch, split3=False), epilogue=epi, name=spec.name,
                          a_param=aname, b_param=bname, c_param=cname, arg_params=arg_params(spec),
                          buffers=tuple(q.name for q in spec.params), operand_dtypes=od,
                          operand_round=role_cast["a"] if f32_cast else A.dtype, direct=not aligned,
                          a_dtype=A.dtype, b_dtype=B.dtype, **split)
    od = tuple((q.name, q.dtype) for q in spec.params if q.dtype in ("f16", "bf16"))
    tiling = choose_tiling(M, N, batch, 32 if b_kmajor else 64)
    return GemmConfig(M=M, N=N, K=K, batch=batch, ab=A.dtype, c=C.dtype, b_kmajor=b_kmajor, **tiling,
                      epilogue=epi, name=spec.name, a_param=aname, b_param=bname, c_param=cname,
                      arg_params=arg_params(spec), buffers=tuple(q.name for q in spec.params),
                      operand_dtypes=od, **split)


def _epilogue_ops(spec, store) -> tuple:
    """The RegStore epilogue Lambda (``mma.py:347-357`` in the reference) as fused ops,
    in statement order: ``copy`` to a 16-bit dtype rounds the accumulator the way
    torch's f16/bf16 matmul result is rounded before the next op; ``relu``; ``add`` of
    a loaded operand (a C-shaped residual, or a bias over N).  Any other Lambda (with
    constants, erf, ...) is lowered statement by statement per element."""
    lam = store.epilogue
    if lam is None:
        return ()
    try:
        return _epilogue_patterns(spec, store)
    except NotImplementedError:
        return (("lambda", lam, _lambda_operands(spec, store), tuple(sorted(spec.constants.items()))),)


def _lambda_operands(spec, store) -> tuple:
    """(load name, kind, buffer) of each buffer the Lambda reads: a C-shaped residual
    or a bias over N (``__N__``, the element's column, in its index)."""
    out = []
    cshape = spec.param(store.dst_buffer).shape
    for s in store.epilogue.body:
        if type(s).__name__ == "Load" and s.input not in spec.constants:
            shape = spec.param(s.input).shape
            if tuple(shape) == tuple(cshape):
                out.append((s.names[0], "residual", s.input))
            elif len(shape) == 1 and shape[0] == cshape[-1]:
                out.append((s.names[0], "bias", s.input))
            else:
                raise NotImplementedError("GEMM epilogue operand shape")
            if spec.param(s.input).dtype not in ("f16", "bf16"):
                raise NotImplementedError("GEMM epilogue operand dtype")
        elif type(s).__name__ not in ("Load", "Assign", "Let"):
            raise NotImplementedError(f"GEMM epilogue statement {type(s).__name__}")
    return tuple(out)


def _epilogue_patterns(spec, store) -> tuple:
    lam = store.epilogue
    ops = []
    loads = {}
    for s in lam.body:
        k = type(s).__name__
        if k == "Load":
            if s.input in spec.constants:
                raise NotImplementedError("GEMM epilogue with constant operands")
            loads[s.names[0]] = s.input
        elif k == "Assign":
            op = s.op.name
            dt = getattr(s.dtype, "name", None)
            if op == "copy":
                if dt in ("f16", "bf16"):
                    ops.append(("round", dt))
            elif op == "relu":
                ops.append(("relu",))
            elif op == "add" and sum(a in loads for a in s.args) == 1:
                buf = loads[[a for a in s.args if a in loads][0]]
                shape = spec.param(buf).shape
                cshape = spec.param(store.dst_buffer).shape
                if tuple(shape) == tuple(cshape):
                    ops.append(("residual", buf))
                elif len(shape) == 1 and shape[0] == cshape[-1]:
                    ops.append(("bias", buf))
                else:
                    raise NotImplementedError("GEMM epilogue operand shape")
            else:
                raise NotImplementedError(f"GEMM epilogue op {op}")
        else:
            raise NotImplementedError(f"GEMM epilogue statement {k}")
    return tuple(ops)


_F32_RATE = {128: 1.0, 64: 0.7, 32: 0.45}


def choose_tiling_f32(M: int, N: int, batch: int, split3: bool = True) -> dict:
    """Tiling of the tf32 GEMM: single CTAs, BN of 128, 64 or 32 by the same
    waves x tile-work estimate as ``choose_tiling``; as many stages as fit (a stage
    holds the f32 tiles, 16 KB + BN x 128 B, and with 3xTF32 their lo parts as much)."""
    best = None
    for bn in (128, 64, 32):
        tiles = batch * (-(-M // 128)) * (-(-N // bn))
        cost = (-(-tiles // SMS)) * 128 * bn / _F32_RATE[bn]
        if best is None or cost < best[0]:
            best = (cost, bn)
    bn = best[1]
    stage = (2 if split3 else 1) * (128 * 128 + bn * 128)
    return {"pair": False, "BN": bn, "stages": min(4, (232448 - 256 - 1024) // stage)}


def analyze_f32(spec) -> GemmConfig:
    """emmy's SIMT matmul family with f32 operands: ``problems/m01_matmul_512`` (a
    cp.async-staged 32x64 CTA tile, ``k_matmul_2967be.ir.txt:1-38``), the split-K form
    with atomic partial sums (``problems/m02_matmul_rect/k_matmul.ir.txt:1-24``),
    ``tests/problems/x_m_*`` (batched, bias + relu and constant-scale tails) and the
    operands cast to bf16 before a product kept exact (``tests/problems/x_q_bf16_mm_t``,
    a warp-shuffle dot product per output, and ``x_q_bf16_mm_odd``, a register tile
    writing split-K partial slices).  Each accumulator adds products of two values
    loaded -- from global memory or from a shared buffer a ``CpAsyncCopy`` filled -- from
    the operands A [.., M, K] and B [.., K, N] (or [.., N, K]), possibly masked to zero
    past the end of K, or adds another such accumulator; the statements between the
    accumulator and the Write of C become the epilogue.  The whole K runs in one pass (a
    split-K ``*_ks`` axis and its atomic adds into the zeroed C, or its partial slices,
    give the same sum), on the 3xTF32 template or, for cast operands, on one exact tf32
    MMA of the rounded values."""
    stmts = list(_walk(spec.body))
    kinds = {type(s).__name__ for s in stmts}
    if kinds & {"MmaSyncPtx", "FragmentRowReduce"}:
        raise NotImplementedError("not the SIMT matmul form")
    accs = [s for s in stmts if type(s).__name__ == "Accum"]
    if not accs:
        raise NotImplementedError("no accumulation")
    order = {id(s): i for i, s in enumerate(stmts)}
    defs = {}
    for s in stmts:
        k = type(s).__name__
        if k == "Load":
            for n in s.names:
                defs[n] = s
        elif k in ("Assign", "Select", "Init"):
            defs[s.name] = s
    staged = {}
    for s in stmts:
        if type(s).__name__ == "CpAsyncCopy":
            if staged.setdefault(s.smem, s.src) != s.src:
                raise NotImplementedError("a shared buffer staged from two sources")

    def source(name):
        """(buffer, Load, cast) of an operand value: copies followed to a Load; a
        narrowing copy (to bf16 / f16) is the IR's cast of the operand."""
        d, cast = defs.get(name), None
        while d is not None and type(d).__name__ == "Assign" and d.op.name == "copy" and len(d.args) == 1:
            dt = getattr(d.dtype, "name", None)
            if dt in ("bf16", "f16"):
                if cast not in (None, dt):
                    raise NotImplementedError("an operand cast twice")
                cast = dt
            d = defs.get(d.args[0])
        if d is None or type(d).__name__ != "Load":
            raise NotImplementedError(f"matmul operand {name} is not a loaded value")
        if d.input in staged:
            return staged[d.input], d, cast
        if d.input in spec.buffers and d.input not in spec.constants:
            return d.input, d, cast
        raise NotImplementedError(f"cannot trace operand {name} to a buffer")

    def is_zero(name):
        d = defs.get(name)
        return d is not None and type(d).__name__ == "Init" and float(d.identity) == 0.0

    def product(name):
        """The multiply an accumulated value is, unwrapping a mask (a Select between the
        product and a zero Init)."""
        d = defs.get(name)
        if d is not None and type(d).__name__ == "Select":
            vals = [br.value for br in d.branches if not is_zero(br.value)]
            if len(vals) != 1 or len(d.branches) < 2:
                raise NotImplementedError("a masked value that is not a product or zero")
            d = defs.get(vals[0])
        if d is None or type(d).__name__ != "Assign" or d.op.name != "multiply" or len(d.args) != 2:
            raise NotImplementedError("an accumulation that is not a sum of products")
        return d

    acc_names = {a.name for a in accs}
    kvars, loads, casts = set(), {}, set()
    for a in accs:
        if a.op.name != "add":
            raise NotImplementedError("an accumulation that is not a sum")
        if a.value in acc_names:          # partial accumulators combined
            continue
        v = product(a.value)
        kvars |= set(a.axes or ())
        for x in v.args:
            buf, ld, cast = source(x)
            loads.setdefault(buf, ld)
            casts.add(cast)
    if len(loads) != 2 or not kvars:
        raise NotImplementedError("products of other than two operands")
    if len(casts) != 1:
        raise NotImplementedError("operands cast differently")
    cast = casts.pop()

    # (writes into shared buffers are the schedule's own combine)
    writes = [s for s in stmts if type(s).__name__ == "Write" and s.output in spec.buffers]
    if not writes or len({w.output for w in writes}) != 1:
        raise NotImplementedError("matmul without a single output")
    first = writes[0]
    cname = first.output
    C = spec.param(cname)
    if len(first.index) < 2 or len(C.shape) < 2:
        raise NotImplementedError("an output without rows and columns")
    rvars, cvars = _vars(first.index[-2]), _vars(first.index[-1])

    def backslice(name):
        """(statements, accumulators) the value ``name`` is computed from."""
        out, seeds, seen = [], set(), set()

        def visit(n):
            if n in acc_names:
                seeds.add(n)
                return
            d = defs.get(n)
            if d is None or type(d).__name__ not in ("Load", "Assign"):
                raise NotImplementedError(f"{n} is not a loaded or computed value")
            if id(d) in seen:
                return
            seen.add(id(d))
            if type(d).__name__ == "Assign":
                for x in d.args:
                    visit(x)
            elif d.input not in spec.constants and d.input not in spec.buffers:
                raise NotImplementedError(f"epilogue reads {d.input}")
            out.append(d)
        visit(name)
        return sorted(out, key=lambda d: order[id(d)]), seeds

    # the epilogue: what the written value is computed from, back to one accumulator;
    # every output element must be computed the same way
    chain, lam_seeds = backslice(first.values[0])

    def signature(c):
        return [(type(d).__name__, getattr(getattr(d, "op", None), "name", None)) for d in c]
    sig = signature(chain)
    for w in writes:
        for val in w.values:
            c, seeds = backslice(val)
            if len(seeds) != 1 or signature(c) != sig:
                raise NotImplementedError("outputs computed from several accumulators or differently")

    def dims(buf, ld):
        """(K dim, free dim, free-dim variables) of an operand, as dims of the global buffer."""
        shape = spec.param(buf).shape
        idx = ld.index
        kd = [i for i, e in enumerate(idx) if _vars(e) & kvars]
        if len(kd) != 1 or len(idx) < 2:
            raise NotImplementedError("K axis not identifiable in an operand index")
        fd = len(idx) - 1 if kd[0] == len(idx) - 2 else len(idx) - 2
        # a staged operand: shared dims are the buffer's trailing dims
        off = len(shape) - len(idx)
        return kd[0] + off, fd + off, _vars(idx[fd])

    (b0, l0), (b1, l1) = loads.items()
    d0, d1 = dims(b0, l0), dims(b1, l1)
    row_only, col_only = rvars - cvars, cvars - rvars
    if d0[2] & row_only and d1[2] & col_only:
        (aname, (ak, af, _)), (bname, (bk, bf, _)) = (b0, d0), (b1, d1)
    elif d1[2] & row_only and d0[2] & col_only:
        (aname, (ak, af, _)), (bname, (bk, bf, _)) = (b1, d1), (b0, d0)
    else:
        raise NotImplementedError("operand roles not identifiable")
    A, B = spec.param(aname), spec.param(bname)
    if A.dtype not in ("f32", "f16", "bf16", "f64") or B.dtype not in ("f32", "f16", "bf16", "f64") or \
            C.dtype not in ("f32", "f64"):
        raise NotImplementedError(f"SIMT matmul {A.dtype} x {B.dtype} -> {C.dtype}")
    if "f64" in (A.dtype, B.dtype) and any(getattr(a.dtype, "name", None) != "f32" for a in accs):
        raise NotImplementedError("f64 products accumulated in f64")
    if cast is None and A.dtype == B.dtype and A.dtype in ("f16", "bf16"):
        cast = A.dtype          # 16-bit operands: exact in tf32, one MMA
    if ak != len(A.shape) - 1:
        raise NotImplementedError("A operand is not K-major")
    b_kmajor = bk == len(B.shape) - 1
    M, K = A.shape[-2], A.shape[-1]
    N = B.shape[bf]
    if B.shape[bk] != K:
        raise NotImplementedError("operand shapes do not form a matmul")
    # emmy's split-K partial slices: a `*_ks` tile axis picks slice ks of an f32
    # [S, .., M, N] buffer that a second kernel sums; the full product goes to slice 0
    tile = spec.body[0] if len(spec.body) == 1 and type(spec.body[0]).__name__ == "Tile" else None
    ks_axes = [ax for ax in (tile.axes if tile else ()) if ax.name.endswith("_ks")]
    cdims, split = tuple(C.shape), {}
    if ks_axes and len(cdims) == len(A.shape) + 1:
        S = int(ks_axes[0].extent.value)
        if len(ks_axes) != 1 or cdims[0] != S or _vars(first.index[0]) != {ks_axes[0].name}:
            raise NotImplementedError("split-K partial slices not addressed by the split axis")
        cdims = cdims[1:]
        split = dict(zero_slots=S - 1, slot_stride=int(math.prod(cdims)))
    if tuple(cdims[-2:]) != (M, N) or not len(A.shape) == len(B.shape) == len(cdims):
        raise NotImplementedError("operand shapes do not form a matmul")
    batch = int(math.prod(cdims[:-2])) if len(cdims) > 2 else 1
    if batch > 1 and (math.prod(A.shape[:-2]) != batch or math.prod(B.shape[:-2]) != batch):
        raise NotImplementedError("broadcast batch operands")
    if any(w.atomic for w in writes) and cname not in spec.zero_outputs:
        raise NotImplementedError("atomic partial sums into an output that is not zeroed")
    # TMA needs f32 operands with 16-byte rows; anything else is fetched by the converters
    direct = A.dtype != "f32" or B.dtype != "f32" or bool((K * 4) % 16 or (not b_kmajor and (N * 4) % 16))

    epi = ()
    if chain:
        if split:
            raise NotImplementedError("an epilogue on split-K partial slices")
        from types import SimpleNamespace
        operands = []
        for d in chain:
            if type(d).__name__ != "Load" or d.input in spec.constants:
                continue
            shape = tuple(spec.param(d.input).shape)
            iv = set().union(*(_vars(e) for e in d.index))
            if shape == tuple(C.shape) and _vars(d.index[-2]) <= rvars and _vars(d.index[-1]) <= cvars:
                operands.append((d.names[0], "residual", d.input))
            elif len(shape) == 1 and shape[0] == N and iv <= cvars:
                operands.append((d.names[0], "bias", d.input))
            else:
                raise NotImplementedError("epilogue operand that is neither a bias over N nor C-shaped")
            if spec.param(d.input).dtype not in ("f32", "f16", "bf16"):
                raise NotImplementedError("epilogue operand dtype")
        lam = SimpleNamespace(params=tuple(lam_seeds), body=tuple(chain), results=(first.values[0],))
        epi = (("lambda", lam, tuple(operands), tuple(sorted(spec.constants.items()))),)
    od = tuple((q.name, q.dtype) for q in spec.params)
    return GemmConfig(M=M, N=N, K=K, batch=batch, ab="f32", c=C.dtype, b_kmajor=b_kmajor,
                      **choose_tiling_f32(M, N, batch, split3=cast is None), epilogue=epi, name=spec.name,
                      a_param=aname, b_param=bname, c_param=cname, arg_params=arg_params(spec),
                      buffers=tuple(q.name for q in spec.params), operand_dtypes=od,
                      operand_round=cast, direct=direct, a_dtype=A.dtype, b_dtype=B.dtype, **split)


def emit_gemm(spec) -> str:
    return emit_gemm_module(analyze(spec))


def emit_gemm_f32(spec) -> str:
    return emit_gemm_module(analyze_f32(spec))
