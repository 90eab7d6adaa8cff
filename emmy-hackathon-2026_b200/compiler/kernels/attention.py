"""Fused attention O = softmax(Q K^T * scale) V on the tcgen05 tensor cores.

Replaces the reference's register-fragment flash attention (``compiler/mma.py``:
``MmaSyncPtx`` for S and O, ``FragmentApply`` scale/exp/rescale, ``FragmentRowReduce``
row max / sum by 2-step shuffles, ``FragmentRepack`` P -> A fragment; K and V read
straight from global memory, ``tests/problems/x_h_attn_128``, ``x_h_sdpa``).

Kernel structure (128 * (NQ + 1) threads, one warpgroup per query tile plus a control
warpgroup).  The CTAs are persistent, one per SM: CTA c takes the units c, c + grid, ...,
a unit being NQ = 2 query tiles of 128 rows of one batch x head (consecutive units share
the batch x head, so concurrent CTAs share K and V in L2; causal: the units with the
most keys first).  Every role loops over its CTA's units: the K / V ring streams on
across unit boundaries, the next unit's Q_t tile is loaded as soon as the last
``Q_t K^T`` of the current unit is done (``q_empty``), the next unit's ``S_t(0)`` are
issued right behind the current unit's last ``O_t += P_t V`` of both tiles, and the
barrier parities count blocks over all units.  Against one CTA per unit this halves
the fixed cost per unit: the same speed at the BASELINE key length (4096), +6.8 % at
2048 keys and +12 % at 1024.  (Issuing a tile's next-unit ``S_t(0)`` straight after its
own last product instead, before the other tile's, measured 4 % slower: the MMA thread
then waits for the next Q tile while the other tile's product is still to be issued.)

* softmax warpgroup t (warps 4t .. 4t+3), one thread per query row (TMEM lane):
  reads its whole 128-key S row out of TMEM in one go (four ``tcgen05.ld.32x32b.x32``,
  one wait), takes the row maximum with three-input ``max``, forms
  ``p = 2^(s*scale*log2e - m)`` (packed ``fma.rn.f32x2`` and ``ex2.approx``, part of
  them optionally on the FMA pipe by a cubic), accumulates the row sum in f32, packs P
  to bf16/f16 and stores it into TMEM over the S columns it has consumed, where the PV
  MMA reads it as its A operand (optionally into a 128B-swizzled K-major shared-memory
  tile instead, which costs the ring two slots).  The running max is updated
  lazily: O (in TMEM) is rescaled only when the max grows by more than 2^8, so most
  blocks skip the correction; the final normalisation by 1/l makes the result exact
  either way.  With two query tiles the control warpgroup hands its registers to the
  softmax warpgroups (``setmaxnreg``), so the S row, the probabilities and the
  addresses stay in registers;
* control warpgroup: warp 4NQ, lane 0 -- TMA: per unit the Q tiles, then K_j and V_j
  (128 keys each) through a ring of 128-byte-swizzled shared-memory slots (as many as
  shared memory holds: 5 at D = 128), full/empty mbarrier per slot; warp 4NQ+1 -- TMEM
  allocation (S_t: 128 f32 columns, O_t: D columns per tile) and, on lane 0, the MMA
  stream: ``S_t = Q_t K_j^T`` (kind::f16, M=128,
  N=128); per tile ``O_t += P_t V_j`` as soon as softmax t hands P_t over, followed by
  ``S_t = Q_t K_{j+1}^T``, so one warpgroup's softmax overlaps the other tile's
  matrix products.  The commit that signals S_t(j+1) also covers O_t += P_t(j) V_j
  (tcgen05 operations of one thread complete in order), so softmax t may reuse its P
  buffer and rescale O_t as soon as it sees S_t(j+1);
* epilogue (softmax warps, per unit): O row from TMEM, times 1/l, to bf16/f16, 128-bit
  stores; the next unit's first ``O_t += P_t V`` overwrites O_t only after softmax t
  has handed over that unit's first P_t, so the read-out needs no barrier of its own.

The online-softmax state (m, l) is f32.  Every mbarrier wait is bounded.  The barrier
protocol is checked under random schedules by ``tests/test_attention_tiles_protocol.py``.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, replace

from ..ptx import Ptx, entry, f32_hex, module
from .common import arg_params, load_pointer, param_symbol
from .gemm import SMS
from .tc import Waits, instr_desc, smem_desc_hi, smem_desc_lo_const

LOG2E = 1.4426950408889634
AB_FORMAT = {"f16": 0, "bf16": 1}
RESCALE_LOG2 = 8.0          # rescale O only when the row max grows by more than 2^8
REGS_CONTROL = 56           # registers per thread left to the control warpgroup (NQ = 2)
MASK_BYTES = {"f16": 2, "bf16": 2, "f32": 4}


@dataclass
class AttnConfig:
    BH: int                  # batch x heads
    Sq: int
    Sk: int
    D: int
    dtype: str = "bf16"
    kt_layout: bool = False  # K given pre-transposed as [.., D, Sk]
    scale: float = 1.0
    name: str = "k_attention"
    q_param: str = "q"
    k_param: str = "k"
    v_param: str = "v"
    o_param: str = "o"
    arg_params: list | None = None
    buffers: tuple = ()
    ring: int | None = None  # K/V ring slots (None: as many as shared memory holds, up to 6)
    poly_every: int = 0      # every n-th probability from the FMA-pipe exp2 (0: all on MUFU)
    p_tmem: bool = True      # P kept in TMEM over the consumed S columns (A operand from TMEM)
    causal: bool = False     # key j > query i masked out (top-left aligned, as is_causal / tril)
    mask_param: str | None = None   # additive score mask buffer, [.., Sq, Sk] row-major
    mask_dtype: str = "f16"
    mask_bh_stride: int = 0  # elements between the masks of consecutive batch x heads (0: shared)
    heads: int = 0           # query heads per batch entry (grouped-query attention; 0: no groups)
    kv_group: int = 1        # query heads per key / value head: head h reads K / V head h // kv_group
    # "tiles": this module's two-tile template; "split_keys": the persistent split-key
    # schedule of attention_split.py (unmasked, non-causal problems only; measured and
    # not the default; EMMY_ATTENTION_SCHEDULE=split_keys selects it wherever it applies)
    schedule: str = "tiles"

    @property
    def BHKV(self) -> int:               # batch x key / value heads
        return self.BH // self.kv_group

    @property
    def DP(self) -> int:                 # head dim padded to whole 64-element swizzle rows
        return -(-self.D // 64) * 64

    @property
    def NQ(self) -> int:
        return 2 if self.Sq > 128 else 1


def register_split(nq: int) -> tuple[int, int, int]:
    """(launch cap, control warpgroup, softmax warpgroups) registers per thread.

    The block is launched with ``cap`` registers per thread (all of the SM's 64K over
    128 * (nq + 1) threads); with two query tiles the control warpgroup gives up all
    but REGS_CONTROL and the softmax warpgroups take them over (``setmaxnreg``).  The
    split never asks for more than the launch holds."""
    nthreads = 128 * (nq + 1)
    cap = min(65536 // nthreads // 8 * 8, 232)
    if nq == 1:
        return cap, cap, cap
    freed = (cap - REGS_CONTROL) * 128
    soft = min(cap + freed // (128 * nq) // 8 * 8, 248)
    assert 128 * REGS_CONTROL + 128 * nq * soft <= nthreads * cap
    return cap, REGS_CONTROL, soft


def emit_attention_module(cfg: AttnConfig) -> str:
    if cfg.schedule == "tiles" and os.environ.get("EMMY_ATTENTION_SCHEDULE") == "split_keys":
        # the whole compile path (bench.py included) on the split-key schedule wherever
        # it applies, for measuring it against this template
        from .attention_split import eligible
        if eligible(cfg):
            cfg = replace(cfg, schedule="split_keys")
    if cfg.schedule == "split_keys":
        from .attention_split import emit_attention_split_module
        return emit_attention_split_module(cfg)
    if cfg.schedule != "tiles":
        raise NotImplementedError(f"attention schedule {cfg.schedule}")
    if cfg.dtype not in AB_FORMAT:
        raise NotImplementedError(f"attention in {cfg.dtype}")
    if cfg.scale <= 0:
        raise NotImplementedError("non-positive softmax scale")
    if cfg.D % 8 or cfg.D > 128:
        raise NotImplementedError(f"head dim {cfg.D}")
    if cfg.kt_layout and cfg.Sk % 8:
        raise NotImplementedError("pre-transposed K rows not 16-byte aligned")
    if cfg.kv_group > 1 and (not cfg.heads or cfg.heads % cfg.kv_group or cfg.BH % cfg.heads):
        raise NotImplementedError("grouped-query attention needs heads divisible by the group")
    p = Ptx()
    NQ, DP = cfg.NQ, cfg.DP
    nblk = -(-cfg.Sk // 128)
    tile_bytes = 128 * DP * 2             # a Q or K or V tile
    p_bytes = 128 * 128 * 2
    smem_cap = 232448 - 512
    R = cfg.ring
    if R is None:
        free = smem_cap - 1024 - NQ * tile_bytes - (0 if cfg.p_tmem else NQ * p_bytes)
        R = max(2, min(6, free // tile_bytes))
    q_off, ring_off = 0, NQ * tile_bytes
    p_off = ring_off + R * tile_bytes
    smem = p_off + (0 if cfg.p_tmem else NQ * p_bytes) + 1024
    if smem > smem_cap:
        raise NotImplementedError("attention tiles exceed shared memory")
    if cfg.mask_param is not None:
        if cfg.mask_dtype not in MASK_BYTES:
            raise NotImplementedError(f"attention mask in {cfg.mask_dtype}")
        if (cfg.Sk * MASK_BYTES[cfg.mask_dtype]) % 16:
            raise NotImplementedError("attention mask rows not 16-byte aligned")
    ncols_used = NQ * (128 + DP)
    ncols = max(32, 1 << math.ceil(math.log2(ncols_used)))
    fmt = AB_FORMAT[cfg.dtype]
    idesc_qk = instr_desc(128, 128, fmt, fmt, False, cfg.kt_layout)
    idesc_pv = instr_desc(128, DP, fmt, fmt, False, True)
    k_sw_hi = smem_desc_hi(1024)
    kmaj_lo = smem_desc_lo_const(16)
    kt_lo = smem_desc_lo_const(DP * 128)        # kt: 64-key blocks of DP d-rows
    v_lo = smem_desc_lo_const(128 * 128)        # V: 64-d blocks of 128 key-rows
    scale_log2 = cfg.scale * LOG2E
    nthreads = 128 * (NQ + 1)
    W_TMA, W_MMA = 4 * NQ, 4 * NQ + 1           # the control warpgroup's working warps
    masked = cfg.Sk % 128 != 0
    cap, regs_ctl, regs_soft = register_split(NQ)

    p.comment(f"tcgen05 attention BH={cfg.BH} Sq={cfg.Sq} Sk={cfg.Sk} D={cfg.D} {cfg.dtype}, "
              f"{NQ} query tiles per CTA, {nblk} key blocks, scale={cfg.scale}")
    ptr = {n: load_pointer(p, n) for n in cfg.buffers}
    status = p.reg("b64")
    p.emit(f"ld.param.u64 {status}, [param__status]\ncvta.to.global.u64 {status}, {status}")
    tq, tk, tv = p.reg("b64"), p.reg("b64"), p.reg("b64")
    for r, n in ((tq, "q"), (tk, "k"), (tv, "v")):
        p.emit(f"mov.u64 {r}, param__tmap_{n}\ncvta.param.u64 {r}, {r}")
    tid, warp, lane = p.regs("u32", 3)
    p.emit(f"mov.u32 {tid}, %tid.x\nshr.u32 {warp}, {tid}, 5\nand.b32 {lane}, {tid}, 31")
    base, bars, abort, tslot = p.regs("u32", 4)
    p.emit(f"""
        mov.u32 {base}, dsmem
        add.u32 {base}, {base}, 1023
        and.b32 {base}, {base}, -1024
        mov.u32 {bars}, gbars
        mov.u32 {abort}, gabort
        mov.u32 {tslot}, gtmem
    """)
    # barrier offsets: per query tile t the Q slot (full / empty), S_t, P_t and O_t;
    # full / empty per ring slot.  (A unit's first O_t += P_t V needs no barrier of its
    # own against the previous unit's epilogue: softmax t reads O_t out before it hands
    # over that unit's first P_t.)
    B_Q = 0
    B_QE = B_Q + 8 * NQ
    B_KVF = B_QE + 8 * NQ
    B_KVE = B_KVF + 8 * R
    B_S = B_KVE + 8 * R
    B_P = B_S + 8 * NQ
    B_O = B_P + 8 * NQ
    nbar = 2 * R + 5 * NQ
    p0 = p.reg("pred")
    l_init = p.label("init_done")
    p.emit(f"setp.ne.u32 {p0}, {tid}, 0\n@{p0} bra {l_init}")
    for t in range(NQ):
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_Q + 8 * t}], 1")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_QE + 8 * t}], 1")
    for s in range(R):
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_KVF + 8 * s}], 1")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_KVE + 8 * s}], 1")
    for t in range(NQ):
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_S + 8 * t}], 1")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_P + 8 * t}], 128")
        p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{B_O + 8 * t}], 1")
    p.emit(f"st.shared.u32 [{abort}], 0\nfence.mbarrier_init.release.cluster\nfence.proxy.async.shared::cta")
    p.place(l_init)
    p1 = p.reg("pred")
    l_alloc = p.label("alloc_done")
    p.emit(f"setp.ne.u32 {p1}, {warp}, {W_MMA}\n@{p1} bra {l_alloc}")
    p.emit(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], {ncols}\n"
           f"tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
    p.place(l_alloc)
    tbase = p.reg("u32")
    p.emit(f"""
        tcgen05.fence::before_thread_sync
        barrier.sync 0
        tcgen05.fence::after_thread_sync
        ld.shared.u32 {tbase}, [{tslot}]
    """)
    waits = Waits(p, status, abort)
    finish = p.label("finish")
    ptrue, pfalse, zr = p.reg("pred"), p.reg("pred"), p.reg("u32")
    p.emit(f"mov.u32 {zr}, 0\nsetp.eq.u32 {ptrue}, {zr}, 0\nsetp.ne.u32 {pfalse}, {zr}, 0")
    # persistent CTAs: unit u = NQ query tiles of one batch x head (bh = u / nqp, first
    # query row 128 NQ (u % nqp); causal: the last tiles, which see the most keys,
    # first); CTA c takes units c, c + grid, ...; nunit = units this CTA takes
    nqp = -(-cfg.Sq // (128 * NQ))
    units = nqp * cfg.BH
    grid = min(SMS, units)
    # (%ctaid.x is read where it is needed, so no register holds it across the loops)

    def unit_coords(ui):
        """(bh, q0, key blocks per tile, key blocks of the unit) of this CTA's ui-th unit."""
        un, bh, q0 = p.regs("u32", 3)
        p.emit(f"mov.u32 {un}, %ctaid.x\nmad.lo.u32 {un}, {ui}, {grid}, {un}\n"
               f"div.u32 {bh}, {un}, {nqp}\nrem.u32 {q0}, {un}, {nqp}")
        if cfg.causal:
            p.emit(f"sub.u32 {q0}, {nqp - 1}, {q0}")
        p.emit(f"mul.lo.u32 {q0}, {q0}, {128 * NQ}")
        # key blocks per query tile: all of them, or (causal) up to the tile's last row
        nbt = []
        for t in range(NQ):
            if cfg.causal:
                r = p.reg("u32")
                p.emit(f"add.u32 {r}, {q0}, {128 * t + 127}\nmin.u32 {r}, {r}, {cfg.Sq - 1}\n"
                       f"shr.u32 {r}, {r}, 7\nadd.u32 {r}, {r}, 1\nmin.u32 {r}, {r}, {nblk}")
                nbt.append(r)
            else:
                nbt.append(str(nblk))
        return bh, q0, nbt, nbt[-1]       # the last tile needs the most blocks

    def unit_loop_end(ui, label):
        """ui += 1; back to ``label`` while this CTA has units left (unit ctaid + ui grid
        exists)."""
        pu, un = p.reg("pred"), p.reg("u32")
        p.emit(f"add.u32 {ui}, {ui}, 1\nmov.u32 {un}, %ctaid.x\nmad.lo.u32 {un}, {ui}, {grid}, {un}\n"
               f"setp.lt.u32 {pu}, {un}, {units}\n@{pu} bra {label}")

    def ring_advance(slot, ph):
        ps = p.reg("pred")
        p.emit(f"add.u32 {slot}, {slot}, 1\nsetp.eq.u32 {ps}, {slot}, {R}\n"
               f"@{ps} mov.u32 {slot}, 0\n@{ps} xor.b32 {ph}, {ph}, 1")

    # -------------------------------------------------------------- role dispatch
    l_ctl, l_soft = p.label("role_control"), p.label("role_softmax")
    pc = p.reg("pred")
    p.emit(f"setp.lt.u32 {pc}, {warp}, {4 * NQ}\n@{pc} bra {l_soft}")
    p.place(l_ctl)
    if NQ == 2:
        p.emit(f"setmaxnreg.dec.sync.aligned.u32 {regs_ctl}")
    l_mma = p.label("role_mma")
    pr, pl = p.reg("pred"), p.reg("pred")
    p.emit(f"setp.ne.u32 {pr}, {warp}, {W_TMA}\n@{pr} bra {l_mma}\nsetp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")

    # ------------------------------------------------------------------ producer
    p.emit(f"prefetch.tensormap [{tq}]\nprefetch.tensormap [{tk}]\nprefetch.tensormap [{tv}]")
    slot, ph, ui = p.regs("u32", 3)
    p.emit(f"mov.u32 {slot}, 0\nmov.u32 {ph}, 0\nmov.u32 {ui}, 0")
    l_punit = p.label("p_unit")
    p.place(l_punit)
    bh, q0, _, nb_cta = unit_coords(ui)
    for t in range(NQ):
        # Q_t's slot is free once the previous unit's last Q_t K^T is done (use ui - 1)
        l_qfree = p.label("p_qfree")
        pq0, qpar = p.reg("pred"), p.reg("u32")
        p.emit(f"setp.eq.u32 {pq0}, {ui}, 0\n@{pq0} bra {l_qfree}\nsub.u32 {qpar}, {ui}, 1\nand.b32 {qpar}, {qpar}, 1")
        waits.wait(_addr(p, bars, B_QE + 8 * t), qpar, "producer", finish)
        p.place(l_qfree)
        qb = _addr(p, bars, B_Q + 8 * t)
        p.emit(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qb}], {tile_bytes}")
        for db in range(DP // 64):
            dst, y = p.reg("u32"), p.reg("u32")
            p.emit(f"add.u32 {dst}, {base}, {q_off + t * tile_bytes + db * 16384}\nadd.u32 {y}, {q0}, {t * 128}")
            p.emit(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                   f"[{dst}], [{tq}, {{{db * 64}, {y}, {bh}}}], [{qb}]")
    kvbh = bh
    if cfg.kv_group > 1:
        # query head h of batch entry b reads key / value head h // g of b
        kvbh, hq = p.reg("u32"), p.reg("u32")
        p.emit(f"div.u32 {kvbh}, {bh}, {cfg.heads}\nrem.u32 {hq}, {bh}, {cfg.heads}\n"
               f"div.u32 {hq}, {hq}, {cfg.kv_group}\nmad.lo.u32 {kvbh}, {kvbh}, {cfg.heads // cfg.kv_group}, {hq}")
    j = p.reg("u32")
    p.emit(f"mov.u32 {j}, 0")
    l_pk = p.label("p_kv")
    p.place(l_pk)
    key0 = p.reg("u32")
    p.emit(f"mul.lo.u32 {key0}, {j}, 128")
    for which in ("k", "v"):
        ea, fa, par, dst0 = p.regs("u32", 4)
        p.emit(f"""
            mad.lo.u32 {ea}, {slot}, 8, {bars}
            add.u32 {fa}, {ea}, {B_KVF}
            add.u32 {ea}, {ea}, {B_KVE}
            xor.b32 {par}, {ph}, 1
        """)
        waits.wait(ea, par, "producer", finish)
        p.emit(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fa}], {tile_bytes}\n"
               f"mad.lo.u32 {dst0}, {slot}, {tile_bytes}, {base}\nadd.u32 {dst0}, {dst0}, {ring_off}")
        if which == "k" and cfg.kt_layout:
            for kb in range(2):
                dst, x = p.reg("u32"), p.reg("u32")
                p.emit(f"add.u32 {dst}, {dst0}, {kb * DP * 128}\nadd.u32 {x}, {key0}, {kb * 64}")
                p.emit(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                       f"[{dst}], [{tk}, {{{x}, 0, {kvbh}}}], [{fa}]")
        else:
            tm = tk if which == "k" else tv
            for db in range(DP // 64):
                dst = p.reg("u32")
                p.emit(f"add.u32 {dst}, {dst0}, {db * 16384}")
                p.emit(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                       f"[{dst}], [{tm}, {{{db * 64}, {key0}, {kvbh}}}], [{fa}]")
        ring_advance(slot, ph)
    pj = p.reg("pred")
    p.emit(f"add.u32 {j}, {j}, 1\nsetp.lt.u32 {pj}, {j}, {nb_cta}\n@{pj} bra {l_pk}")
    unit_loop_end(ui, l_punit)
    p.emit(f"bra {finish}")

    # ----------------------------------------------------------------------- MMA
    p.place(l_mma)
    p.emit(f"setp.ne.u32 {pr}, {warp}, {W_MMA}\n@{pr} bra {finish}\nsetp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")
    cslot, cph, ui = p.regs("u32", 3)
    p.emit(f"mov.u32 {cslot}, 0\nmov.u32 {cph}, 0\nmov.u32 {ui}, 0")
    cntp = [p.reg("u32") for _ in range(NQ)]      # P_t hand-overs taken so far, all units
    for r in cntp:
        p.emit(f"mov.u32 {r}, 0")

    def wait_slot(sl, ph_):
        fa = p.reg("u32")
        p.emit(f"mad.lo.u32 {fa}, {sl}, 8, {bars}\nadd.u32 {fa}, {fa}, {B_KVF}")
        waits.wait(fa, ph_, "mma", finish)
        p.emit("tcgen05.fence::after_thread_sync")

    def release_slot(sl):
        ea = p.reg("u32")
        p.emit(f"mad.lo.u32 {ea}, {sl}, 8, {bars}\nadd.u32 {ea}, {ea}, {B_KVE}")
        p.emit(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{ea}]")

    def desc(addr_reg, lo_const, hi_const):
        lo, d = p.reg("u32"), p.reg("b64")
        p.emit(f"shr.u32 {lo}, {addr_reg}, 4\nor.b32 {lo}, {lo}, {lo_const}\nmov.b64 {d}, {{{lo}, {hi_const}}}")
        return d

    def issue_qk(t, sl):
        """S_t = Q_t K^T over the DP head-dim (K steps of 16)."""
        kbase, qa, ka = p.reg("u32"), p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {kbase}, {sl}, {tile_bytes}, {base}\nadd.u32 {kbase}, {kbase}, {ring_off}")
        st = p.reg("u32")
        p.emit(f"add.u32 {st}, {tbase}, {t * 128}")
        for kk in range(DP // 16):
            p.emit(f"add.u32 {qa}, {base}, {q_off + t * tile_bytes + (kk // 4) * 16384 + (kk % 4) * 32}")
            if cfg.kt_layout:
                p.emit(f"add.u32 {ka}, {kbase}, {kk * 2048}")
                kd = desc(ka, kt_lo, k_sw_hi)
            else:
                p.emit(f"add.u32 {ka}, {kbase}, {(kk // 4) * 16384 + (kk % 4) * 32}")
                kd = desc(ka, kmaj_lo, k_sw_hi)
            qd = desc(qa, kmaj_lo, k_sw_hi)
            pe = pfalse if kk == 0 else ptrue
            p.emit(f"tcgen05.mma.cta_group::1.kind::f16 [{st}], {qd}, {kd}, {idesc_qk}, {pe}")
        sb = p.reg("u32")
        p.emit(f"add.u32 {sb}, {bars}, {B_S + 8 * t}\n"
               f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{sb}]")

    def issue_pv(t, sl, first_block_pred):
        """O_t (+)= P_t V over the 128 keys of the block."""
        vbase, pa, va = p.reg("u32"), p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {vbase}, {sl}, {tile_bytes}, {base}\nadd.u32 {vbase}, {vbase}, {ring_off}")
        ot = p.reg("u32")
        p.emit(f"add.u32 {ot}, {tbase}, {NQ * 128 + t * DP}")
        for kk in range(128 // 16):
            p.emit(f"add.u32 {va}, {vbase}, {kk * 2048}")
            vd = desc(va, v_lo, k_sw_hi)
            if kk == 0:
                pe = p.reg("pred")
                p.emit(f"not.pred {pe}, {first_block_pred}")
            else:
                pe = ptrue
            if cfg.p_tmem:
                # A = P from TMEM: 16 keys of bf16/f16 pairs = 8 columns per K step
                p.emit(f"add.u32 {pa}, {tbase}, {t * 128 + kk * 8}")
                p.emit(f"tcgen05.mma.cta_group::1.kind::f16 [{ot}], [{pa}], {vd}, {idesc_pv}, {pe}")
            else:
                p.emit(f"add.u32 {pa}, {base}, {p_off + t * p_bytes + (kk // 4) * 16384 + (kk % 4) * 32}")
                pd = desc(pa, kmaj_lo, k_sw_hi)
                p.emit(f"tcgen05.mma.cta_group::1.kind::f16 [{ot}], {pd}, {vd}, {idesc_pv}, {pe}")
        ob = p.reg("u32")
        p.emit(f"add.u32 {ob}, {bars}, {B_O + 8 * t}\n"
               f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{ob}]")

    def q_release_if_last(t, blk):
        """Q_t's slot is free for the next unit once its last Q_t K^T (block nbt_t - 1) is
        done; ``blk`` (a register or a constant) is the block whose Q_t K^T was just issued."""
        l_keep = None
        if cfg.causal:
            l_keep, plast, last = p.label("m_qkeep"), p.reg("pred"), p.reg("u32")
            p.emit(f"sub.u32 {last}, {nbt[t]}, 1\nsetp.ne.u32 {plast}, {last}, {blk}\n@{plast} bra {l_keep}")
        elif nblk == 1:
            pass                                    # every Q_t K^T is the unit's last
        elif isinstance(blk, int):
            if blk != nblk - 1:
                return
        else:
            l_keep, plast = p.label("m_qkeep"), p.reg("pred")
            p.emit(f"setp.ne.u32 {plast}, {blk}, {nblk - 1}\n@{plast} bra {l_keep}")
        p.emit(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
               f"[{_addr(p, bars, B_QE + 8 * t)}]")
        if l_keep is not None:
            p.place(l_keep)
    l_munit = p.label("m_unit")
    p.place(l_munit)
    _, _, nbt, nb_cta = unit_coords(ui)
    upar = p.reg("u32")
    p.emit(f"and.b32 {upar}, {ui}, 1")
    # unit prologue: S_t(0) once this unit's Q_t is in (B_Q[t], use ui); on an SM the
    # previous unit's O_t += P_t V were issued before, so they complete first
    kslot, kph = p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {kslot}, {cslot}\nmov.u32 {kph}, {cph}")
    wait_slot(kslot, kph)
    for t in range(NQ):
        waits.wait(_addr(p, bars, B_Q + 8 * t), upar, "mma", finish)
        p.emit("tcgen05.fence::after_thread_sync")
        issue_qk(t, kslot)
        q_release_if_last(t, 0)
    release_slot(kslot)
    ring_advance(cslot, cph)
    jm = p.reg("u32")
    p.emit(f"mov.u32 {jm}, 0")
    l_mj = p.label("m_blk")
    p.place(l_mj)
    vslot, vph = p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {vslot}, {cslot}\nmov.u32 {vph}, {cph}")
    ring_advance(cslot, cph)
    wait_slot(vslot, vph)
    pfirst, pmore = p.reg("pred"), p.reg("pred")
    nxt = p.reg("u32")
    p.emit(f"setp.eq.u32 {pfirst}, {jm}, 0\nadd.u32 {nxt}, {jm}, 1\nsetp.lt.u32 {pmore}, {nxt}, {nb_cta}")
    p.emit(f"mov.u32 {kslot}, {cslot}\nmov.u32 {kph}, {cph}")
    kwait = p.reg("pred")                  # K_{j+1} not yet waited for in this block
    p.emit(f"mov.pred {kwait}, {ptrue}")
    for t in range(NQ):
        l_tdone = p.label("m_tdone")
        if cfg.causal and t < NQ - 1:
            pact = p.reg("pred")           # (causal) this tile may stop before the CTA does
            p.emit(f"setp.lt.u32 {pact}, {jm}, {nbt[t]}\n@!{pact} bra {l_tdone}")
        pb, pph = p.reg("u32"), p.reg("u32")
        p.emit(f"add.u32 {pb}, {bars}, {B_P + 8 * t}\nand.b32 {pph}, {cntp[t]}, 1\nadd.u32 {cntp[t]}, {cntp[t]}, 1")
        waits.wait(pb, pph, "mma", finish)
        p.emit("tcgen05.fence::after_thread_sync")
        issue_pv(t, vslot, pfirst)
        pm_t = pmore
        if cfg.causal and t < NQ - 1:
            pm_t = p.reg("pred")
            p.emit(f"setp.lt.u32 {pm_t}, {nxt}, {nbt[t]}")
        skip = p.label("m_noqk")
        p.emit(f"@!{pm_t} bra {skip}")
        l_kw = p.label("m_kwaited")
        p.emit(f"@!{kwait} bra {l_kw}")
        wait_slot(kslot, kph)
        p.emit(f"mov.pred {kwait}, {pfalse}")
        p.place(l_kw)
        issue_qk(t, kslot)
        q_release_if_last(t, nxt)
        p.place(skip)
        p.place(l_tdone)
    release_slot(vslot)
    l_norel = p.label("m_norel")
    p.emit(f"@!{pmore} bra {l_norel}")
    release_slot(kslot)
    ring_advance(cslot, cph)
    p.place(l_norel)
    p.emit(f"mov.u32 {jm}, {nxt}\n@{pmore} bra {l_mj}")
    unit_loop_end(ui, l_munit)
    p.emit(f"bra {finish}")

    # ------------------------------------------------------------------ softmax
    p.place(l_soft)
    if NQ == 2:
        p.emit(f"setmaxnreg.inc.sync.aligned.u32 {regs_soft}")
    _emit_softmax(p, cfg, ptr, bars, B_S, B_P, B_O, tbase, base, p_off, p_bytes, warp, lane,
                  unit_coords, unit_loop_end, scale_log2, masked, waits, finish)

    # ------------------------------------------------------------------- finish
    p.place(finish)
    pw1 = p.reg("pred")
    done = p.label("done")
    p.emit(f"""
        tcgen05.fence::before_thread_sync
        barrier.sync 0
        tcgen05.fence::after_thread_sync
        setp.ne.u32 {pw1}, {warp}, {W_MMA}
        @{pw1} bra {done}
        bar.warp.sync -1
        tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tbase}, {ncols}
    """)
    p.place(done)
    p.emit("ret")

    params = list(cfg.arg_params or [f".param .u64 {param_symbol(n)}" for n in cfg.buffers])
    params += [".param .align 64 .b8 param__tmap_q[128]", ".param .align 64 .b8 param__tmap_k[128]",
               ".param .align 64 .b8 param__tmap_v[128]", ".param .u64 param__status"]
    # one CTA per SM (its shared memory allows no more): the launch takes the whole
    # register file, which setmaxnreg then redistributes between the warpgroups
    text = entry(cfg.name, params, p, maxntid=nthreads, extra_directives=f"\n.maxnreg {cap}")
    statics = (f"\t.shared .align 8 .b64 gbars[{nbar}];\n\t.shared .align 4 .u32 gabort;\n"
               f"\t.shared .align 4 .u32 gtmem;\n")
    text = text.replace("{\n", "{\n" + statics, 1)
    eb = 2
    # (query, key) pairs that take part: all of them, or (causal) key <= query
    visible = (sum(min(r + 1, cfg.Sk) for r in range(cfg.Sq)) if cfg.causal else cfg.Sq * cfg.Sk)
    kmap = ({"dims": [cfg.Sk, cfg.D, cfg.BHKV], "strides": [cfg.Sk * eb, cfg.D * cfg.Sk * eb],
             "box": [64, DP, 1]} if cfg.kt_layout else
            {"dims": [cfg.D, cfg.Sk, cfg.BHKV], "strides": [cfg.D * eb, cfg.Sk * cfg.D * eb],
             "box": [64, 128, 1]})
    launch = {
        "kind": "attention", "grid": [grid, 1, 1], "block": [nthreads, 1, 1],
        "cluster": [1, 1, 1], "smem": smem, "flops": 4 * cfg.BH * visible * cfg.D,
        "exps": cfg.BH * visible,
        "extra_params": [
            {"kind": "tmap", "buffer": cfg.q_param, "dtype": cfg.dtype, "dims": [cfg.D, cfg.Sq, cfg.BH],
             "strides": [cfg.D * eb, cfg.Sq * cfg.D * eb], "box": [64, 128, 1], "swizzle": 128},
            {"kind": "tmap", "buffer": cfg.k_param, "dtype": cfg.dtype, "swizzle": 128, **kmap},
            {"kind": "tmap", "buffer": cfg.v_param, "dtype": cfg.dtype, "dims": [cfg.D, cfg.Sk, cfg.BHKV],
             "strides": [cfg.D * eb, cfg.Sk * cfg.D * eb], "box": [64, 128, 1], "swizzle": 128},
            {"kind": "status"},
        ],
    }
    return module([text], launch, globals_=[".extern .shared .align 1024 .b8 dsmem[];"])


# 2^f on f in [-1/2, 1/2]: cubic fitted here by least squares on the relative error
# (iteratively reweighted towards minimax); max relative error 7.7e-5, far below the
# bf16 rounding the probabilities get next.
EXP2_POLY = (0.9999262094497681, 0.6932613253593445, 0.2426345944404602, 0.05518098175525665)


def emit_exp2_poly(p: Ptx, dst: str, x: str) -> None:
    """2^x on the FMA/ALU pipes (Cody-Waite split): j = round(x) by adding 1.5*2^23,
    f = x - j in [-1/2, 1/2], 2^f by the cubic, and 2^j by adding j to the exponent
    field.  x is clamped at -125 so the exponent arithmetic stays in range."""
    xc, t, jf, f, q = p.regs("f32", 5)
    tb, qb = p.reg("b32"), p.reg("b32")
    c0, c1, c2, c3 = (f32_hex(c) for c in EXP2_POLY)
    p.emit(f"""
        max.f32 {xc}, {x}, 0fC2FA0000
        add.rn.f32 {t}, {xc}, 0f4B400000
        sub.rn.f32 {jf}, {t}, 0f4B400000
        sub.rn.f32 {f}, {xc}, {jf}
        fma.rn.f32 {q}, {f}, {c3}, {c2}
        fma.rn.f32 {q}, {q}, {f}, {c1}
        fma.rn.f32 {q}, {q}, {f}, {c0}
        mov.b32 {tb}, {t}
        shl.b32 {tb}, {tb}, 23
        mov.b32 {qb}, {q}
        add.s32 {qb}, {qb}, {tb}
        mov.b32 {dst}, {qb}
    """)


def _addr(p: Ptx, base: str, off: int) -> str:
    r = p.reg("u32")
    p.emit(f"add.u32 {r}, {base}, {off}")
    return r


def _max_tree(p: Ptx, vals: list) -> str:
    """Maximum of ``vals`` by a tree of three-input ``max.f32``."""
    red = list(vals)
    while len(red) > 1:
        nxt = []
        i = 0
        while i < len(red):
            if len(red) - i >= 3:
                r = p.reg("f32")
                p.emit(f"max.f32 {r}, {red[i]}, {red[i + 1]}, {red[i + 2]}")
                i += 3
            elif len(red) - i == 2:
                r = p.reg("f32")
                p.emit(f"max.f32 {r}, {red[i]}, {red[i + 1]}")
                i += 2
            else:
                r = red[i]
                i += 1
            nxt.append(r)
        red = nxt
    return red[0]


def _add_mask(p: Ptx, cfg: AttnConfig, fv: list, mrow: str, jj: str, scale_log2: float) -> None:
    """fv[i] <- fv[i] * scale*log2e + mask[row, 128 jj + i] * log2e for the block's 128
    keys; 16-byte loads, none past the row's end (keys >= Sk are masked afterwards)."""
    esz = MASK_BYTES[cfg.mask_dtype]
    per = 16 // esz                       # mask values per 16-byte load
    a = p.reg("b64")
    kb = p.reg("u32")
    p.emit(f"mul.wide.u32 {a}, {jj}, {128 * esz}\nadd.s64 {a}, {a}, {mrow}\nmul.lo.u32 {kb}, {jj}, 128")
    l2e = f32_hex(LOG2E)
    sl = f32_hex(scale_log2)
    for v in range(128 // per):
        w = [p.reg("b32") for _ in range(4)]
        pin, kx = p.reg("pred"), p.reg("u32")
        p.emit(f"add.u32 {kx}, {kb}, {v * per}\nsetp.lt.u32 {pin}, {kx}, {cfg.Sk}")
        for r in w:
            p.emit(f"mov.b32 {r}, 0")
        p.emit(f"@{pin} ld.global.nc.v4.b32 {{{', '.join(w)}}}, [{a}+{v * 16}]")
        vals = []
        for r in w:
            if esz == 4:
                f = p.reg("f32")
                p.emit(f"mov.b32 {f}, {r}")
                vals.append(f)
                continue
            lo, hi = p.reg("f32"), p.reg("f32")
            if cfg.mask_dtype == "f16":
                h0, h1 = p.reg("b16"), p.reg("b16")
                p.emit(f"mov.b32 {{{h0}, {h1}}}, {r}\ncvt.f32.f16 {lo}, {h0}\ncvt.f32.f16 {hi}, {h1}")
            else:                         # bf16: the high half of an f32
                bl, bh_ = p.reg("b32"), p.reg("b32")
                p.emit(f"shl.b32 {bl}, {r}, 16\nand.b32 {bh_}, {r}, -65536\n"
                       f"mov.b32 {lo}, {bl}\nmov.b32 {hi}, {bh_}")
            vals += [lo, hi]
        for k, mval in enumerate(vals):
            i = v * per + k
            ms = p.reg("f32")
            p.emit(f"mul.rn.f32 {ms}, {mval}, {l2e}\nfma.rn.f32 {fv[i]}, {fv[i]}, {sl}, {ms}")


def _emit_softmax(p: Ptx, cfg: AttnConfig, ptr, bars, B_S, B_P, B_O, tbase, base, p_off, p_bytes,
                  warp, lane, unit_coords, unit_loop_end, scale_log2, masked, waits: Waits, finish):
    NQ, DP = cfg.NQ, cfg.DP
    t, q, row, lanebits = p.regs("u32", 4)
    # warps 0..3 -> tile 0, 4..7 -> tile 1; TMEM lane quarter = warp % 4
    p.emit(f"""
        shr.u32 {t}, {warp}, 2
        and.b32 {q}, {warp}, 3
        mad.lo.u32 {row}, {q}, 32, {lane}
        shl.b32 {lanebits}, {q}, 21
    """)
    s_ta, o_ta = p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {s_ta}, {t}, 128, {tbase}
        add.u32 {s_ta}, {s_ta}, {lanebits}
        mad.lo.u32 {o_ta}, {t}, {DP}, {tbase}
        add.u32 {o_ta}, {o_ta}, {NQ * 128}
        add.u32 {o_ta}, {o_ta}, {lanebits}
    """)
    sbar, pbar, obar = p.regs("u32", 3)
    p.emit(f"""
        mad.lo.u32 {sbar}, {t}, 8, {bars}
        add.u32 {pbar}, {sbar}, {B_P}
        add.u32 {obar}, {sbar}, {B_O}
        add.u32 {sbar}, {sbar}, {B_S}
    """)
    # this thread's P row in smem: tile t, row r; 16-byte chunk c of a 64-key block
    # lives at chunk (c ^ (r % 8)) of the row (128-byte swizzle)
    chunk_addr = {}
    if not cfg.p_tmem:
        prow, rx = p.reg("u32"), p.reg("u32")
        p.emit(f"""
            mad.lo.u32 {prow}, {t}, {p_bytes}, {base}
            add.u32 {prow}, {prow}, {p_off}
            mad.lo.u32 {prow}, {row}, 128, {prow}
            and.b32 {rx}, {row}, 7
        """)
        for c16 in range(16):            # 16 chunks of 8 keys = 128 keys
            blk, c = c16 // 8, c16 % 8
            a = p.reg("u32")
            p.emit(f"xor.b32 {a}, {rx}, {c}\nmad.lo.u32 {a}, {a}, 16, {prow}\nadd.u32 {a}, {a}, {blk * 16384}")
            chunk_addr[c16] = a
    cvt = "cvt.rn.bf16x2.f32" if cfg.dtype == "bf16" else "cvt.rn.f16x2.f32"
    sl2, slr = p.reg("b64"), p.reg("f32")
    pre_scaled = cfg.mask_param is not None
    p.emit(f"mov.f32 {slr}, {f32_hex(1.0 if pre_scaled else scale_log2)}\nmov.b64 {sl2}, {{{slr}, {slr}}}")
    # persistent: this CTA's units one after the other; gcnt = S_t hand-overs so far
    ui, gcnt = p.regs("u32", 2)
    p.emit(f"mov.u32 {ui}, 0\nmov.u32 {gcnt}, 0")
    l_sunit = p.label("s_unit")
    p.place(l_sunit)
    bh, q0, nbt, _ = unit_coords(ui)
    # this tile's number of key blocks and this thread's query row
    if len(set(nbt)) == 1:
        nbm = nbt[0]
    else:
        nbm, pt0 = p.reg("u32"), p.reg("pred")
        p.emit(f"setp.eq.u32 {pt0}, {t}, 0\nselp.b32 {nbm}, {nbt[0]}, {nbt[1]}, {pt0}")
    qrow = p.reg("u32")
    p.emit(f"mad.lo.u32 {qrow}, {t}, 128, {q0}\nadd.u32 {qrow}, {qrow}, {row}")
    mrow = None
    if cfg.mask_param is not None:
        # this row of the additive mask: mask[bh, min(qrow, Sq - 1), :]
        esz = MASK_BYTES[cfg.mask_dtype]
        mrow, w64, qc = p.reg("b64"), p.reg("b64"), p.reg("u32")
        p.emit(f"""
            min.u32 {qc}, {qrow}, {cfg.Sq - 1}
            mul.wide.u32 {mrow}, {bh}, {cfg.mask_bh_stride * esz}
            mul.wide.u32 {w64}, {qc}, {cfg.Sk * esz}
            add.s64 {mrow}, {mrow}, {w64}
            add.s64 {mrow}, {mrow}, {ptr[cfg.mask_param]}
        """)
    m, l = p.reg("f32"), p.reg("f32")
    p.emit(f"mov.f32 {m}, 0fF149F2CA\nmov.f32 {l}, 0f00000000")     # m = -1e30 (log2 domain)
    jj = p.reg("u32")
    p.emit(f"mov.u32 {jj}, 0")
    l_blk = p.label("s_blk")
    p.place(l_blk)
    par = p.reg("u32")
    p.emit(f"and.b32 {par}, {gcnt}, 1")
    # S_t(j) complete; its commit also covers O_t += P_t(j-1) V_{j-1}, so the P buffer
    # is free and O_t holds every earlier block
    waits.wait(sbar, par, "softmax", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    # the whole S row in registers: four loads in flight, one wait; masked and scaled as
    # the score chain says
    fv = [p.reg("f32") for _ in range(128)]
    keyb = None
    if masked:
        keyb = p.reg("u32")
        p.emit(f"mul.lo.u32 {keyb}, {jj}, 128")

    def load_s():
        sv = [p.reg("b32") for _ in range(128)]
        for c in range(4):
            p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(sv[32 * c:32 * c + 32])}}}, "
                   f"[{s_ta}+{c * 32}]")
        p.emit("tcgen05.wait::ld.sync.aligned")
        for i in range(128):
            p.emit(f"mov.b32 {fv[i]}, {sv[i]}")
        if cfg.mask_param is not None:
            # scores in the log2 domain with the additive mask: s*scale*log2e + mask*log2e
            _add_mask(p, cfg, fv, mrow, jj, scale_log2)
        if masked:
            for i in range(128):
                pk, kx = p.reg("pred"), p.reg("u32")
                p.emit(f"add.u32 {kx}, {keyb}, {i}\nsetp.ge.u32 {pk}, {kx}, {cfg.Sk}\n"
                       f"@{pk} mov.f32 {fv[i]}, 0fFF800000")
        if cfg.causal:
            # keys past this thread's query row are out: key 128 jj + i > qrow <=> i > lim
            lim, pneed, pany_c = p.reg("u32"), p.reg("pred"), p.reg("pred")
            l_nocausal = p.label("s_nocausal")
            p.emit(f"""
                mad.lo.s32 {lim}, {jj}, -128, {qrow}
                setp.lt.s32 {pneed}, {lim}, 127
                vote.sync.any.pred {pany_c}, {pneed}, -1
                @!{pany_c} bra {l_nocausal}
            """)
            for i in range(128):
                pk = p.reg("pred")
                p.emit(f"setp.lt.s32 {pk}, {lim}, {i}\n@{pk} mov.f32 {fv[i]}, 0fFF800000")
            p.place(l_nocausal)

    # the packed P chunks and the chunks' row sums, stored / added once the row is done
    packed = [[p.reg("b32") for _ in range(16)] for _ in range(4)]
    psum = [p.reg("f32") for _ in range(4)]

    def exps():
        """p = 2^(s*scale*log2e - m) per 32-key chunk, its row sum and bf16/f16 pack."""
        negm, nm2 = p.reg("f32"), p.reg("b64")
        p.emit(f"neg.f32 {negm}, {m}\nmov.b64 {nm2}, {{{negm}, {negm}}}")
        for c in range(4):
            ps = []
            for i in range(32 * c, 32 * c + 32, 2):
                x2, e2 = p.reg("b64"), p.reg("b64")
                ea, eb = p.reg("f32"), p.reg("f32")
                p.emit(f"mov.b64 {x2}, {{{fv[i]}, {fv[i + 1]}}}\n"
                       f"fma.rn.f32x2 {e2}, {x2}, {sl2}, {nm2}\nmov.b64 {{{ea}, {eb}}}, {e2}")
                for k, e in ((i, ea), (i + 1, eb)):
                    if cfg.poly_every and not masked and k % cfg.poly_every == cfg.poly_every - 1:
                        emit_exp2_poly(p, e, e)     # offload part of the exponentials from MUFU
                    else:
                        p.emit(f"ex2.approx.ftz.f32 {e}, {e}")
                    ps.append(e)
            # row sum: pairwise f32x2 adds, then the two halves
            red = []
            for i in range(0, 32, 2):
                r = p.reg("b64")
                p.emit(f"mov.b64 {r}, {{{ps[i]}, {ps[i + 1]}}}")
                red.append(r)
            while len(red) > 1:
                nxt = []
                for i in range(0, len(red), 2):
                    r = p.reg("b64")
                    p.emit(f"add.rn.f32x2 {r}, {red[i]}, {red[i + 1]}")
                    nxt.append(r)
                red = nxt
            h1 = p.reg("f32")
            p.emit(f"mov.b64 {{{psum[c]}, {h1}}}, {red[0]}\nadd.rn.f32 {psum[c]}, {psum[c]}, {h1}")
            for i in range(16):
                p.emit(f"{cvt} {packed[c][i]}, {ps[2 * i + 1]}, {ps[2 * i]}")

    def o_correction(alpha):
        """O *= alpha (the whole warp, when any of its rows moved its maximum)."""
        ov = [p.reg("b32") for _ in range(32)]
        for c in range(DP // 32):
            p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{o_ta}+{c * 32}]")
            p.emit("tcgen05.wait::ld.sync.aligned")
            for i in range(32):
                f = p.reg("f32")
                p.emit(f"mov.b32 {f}, {ov[i]}\nmul.rn.f32 {f}, {f}, {alpha}\nmov.b32 {ov[i]}, {f}")
            p.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{o_ta}+{c * 32}], {{{', '.join(ov)}}}")
        p.emit("tcgen05.wait::st.sync.aligned")

    def block_max(vals_max):
        mx = p.reg("f32")
        p.emit(f"mov.f32 {mx}, {vals_max}")
        if cfg.mask_param is None:
            p.emit(f"mul.rn.f32 {mx}, {mx}, {f32_hex(scale_log2)}")
        return mx

    load_s()
    pfirst = p.reg("pred")
    p.emit(f"setp.eq.u32 {pfirst}, {jj}, 0")
    mx = block_max(_max_tree(p, fv))
    mn, alpha, thr = p.reg("f32"), p.reg("f32"), p.reg("f32")
    prs = p.reg("pred")
    p.emit(f"""
        max.f32 {mn}, {m}, {mx}
        add.rn.f32 {thr}, {m}, {f32_hex(RESCALE_LOG2)}
        setp.gt.f32 {prs}, {mn}, {thr}
        @{pfirst} mov.f32 {m}, {mn}
        mov.f32 {alpha}, 0f3F800000
    """)
    # (first block: m takes the block max; later blocks rescale only past the threshold)
    d0, pnf = p.reg("f32"), p.reg("pred")
    p.emit(f"""
        not.pred {pnf}, {pfirst}
        and.pred {prs}, {prs}, {pnf}
        sub.rn.f32 {d0}, {m}, {mn}
        @{prs} ex2.approx.ftz.f32 {alpha}, {d0}
        @{prs} mov.f32 {m}, {mn}
        mul.rn.f32 {l}, {l}, {alpha}
    """)
    # lazy O correction: the whole warp takes part when any of its rows needs it
    pany = p.reg("pred")
    l_nores = p.label("s_nores")
    p.emit(f"vote.sync.any.pred {pany}, {prs}, -1\n@!{pany} bra {l_nores}")
    o_correction(alpha)
    p.place(l_nores)
    exps()
    tot, t23 = p.reg("f32"), p.reg("f32")
    p.emit(f"add.rn.f32 {tot}, {psum[0]}, {psum[1]}\nadd.rn.f32 {t23}, {psum[2]}, {psum[3]}\n"
           f"add.rn.f32 {tot}, {tot}, {t23}\nadd.rn.f32 {l}, {l}, {tot}")
    for c in range(4):
        if cfg.p_tmem:
            # P chunk c (32 keys = 16 packed columns) over the S columns read
            p.emit(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{s_ta}+{c * 16}], {{{', '.join(packed[c])}}}")
        else:
            for g in range(4):
                c16 = c * 4 + g
                p.emit(f"st.shared.v4.b32 [{chunk_addr[c16]}], {{{', '.join(packed[c][4 * g:4 * g + 4])}}}")
    if cfg.p_tmem:
        p.emit("tcgen05.wait::st.sync.aligned")
    else:
        p.emit("fence.proxy.async.shared::cta")
    p.emit(f"""
        tcgen05.fence::before_thread_sync
        mbarrier.arrive.shared::cta.b64 _, [{pbar}]
        add.u32 {jj}, {jj}, 1
        add.u32 {gcnt}, {gcnt}, 1
    """)
    pj = p.reg("pred")
    p.emit(f"setp.lt.u32 {pj}, {jj}, {nbm}\n@{pj} bra {l_blk}")
    # epilogue: O / l once the last O_t += P_t V has landed
    parf = p.reg("u32")
    p.emit(f"sub.u32 {parf}, {gcnt}, 1\nand.b32 {parf}, {parf}, 1")
    waits.wait(obar, parf, "softmax", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    inv = p.reg("f32")
    p.emit(f"rcp.rn.f32 {inv}, {l}")
    grow, prow_ok = qrow, p.reg("pred")
    bh, _, _, _ = unit_coords(ui)
    p.emit(f"setp.lt.u32 {prow_ok}, {grow}, {cfg.Sq}")
    oadr, w64 = p.reg("b64"), p.reg("b64")
    p.emit(f"""
        mul.wide.u32 {oadr}, {bh}, {cfg.Sq}
        cvt.u64.u32 {w64}, {grow}
        add.s64 {oadr}, {oadr}, {w64}
        mul.lo.s64 {oadr}, {oadr}, {cfg.D * 2}
        add.s64 {oadr}, {oadr}, {ptr[cfg.o_param]}
    """)
    ov = [p.reg("b32") for _ in range(32)]
    for c in range(DP // 32):
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{o_ta}+{c * 32}]")
        p.emit("tcgen05.wait::ld.sync.aligned")
        if c * 32 >= cfg.D:
            continue
        fs = []
        for i in range(32):
            f = p.reg("f32")
            p.emit(f"mov.b32 {f}, {ov[i]}\nmul.rn.f32 {f}, {f}, {inv}")
            fs.append(f)
        packed = [p.reg("b32") for _ in range(16)]
        for i in range(16):
            p.emit(f"{cvt} {packed[i]}, {fs[2 * i + 1]}, {fs[2 * i]}")
        for g in range(4):
            if c * 32 + 8 * g >= cfg.D:
                break
            p.emit(f"@{prow_ok} st.global.v4.b32 [{oadr}+{(c * 32 + 8 * g) * 2}], "
                   f"{{{', '.join(packed[4 * g:4 * g + 4])}}}")
    # (every O_t load above has completed: the next unit's first P_t hand-over, after
    # which O_t is overwritten, comes later in this thread)
    unit_loop_end(ui, l_sunit)
    p.emit(f"bra {finish}")


# ---------------------------------------------------------------------------
# recognising the IR's attention family


def _walk(body):
    for s in body:
        yield s
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple):
                yield from _walk(sub)


def _frag_base(name: str) -> str:
    """``_qa0_[_r2]`` -> ``_qa0_``, ``_kb[_r0]`` -> ``_kb``."""
    return name.split("[")[0]


def analyze(spec) -> AttnConfig:
    from ..stmts import expr_vars
    stmts = list(_walk(spec.body))
    kinds = {type(s).__name__ for s in stmts}
    if "FragmentRowReduce" not in kinds or "MmaSyncPtx" not in kinds:
        raise NotImplementedError("not a tensor-core attention")
    ldm = [s for s in stmts if type(s).__name__ == "LdmatrixLoad"]
    frag_src = {}
    for s in ldm:
        frag_src.setdefault(_frag_base(s.frag), s)
        if s.pair_frag:
            frag_src.setdefault(_frag_base(s.pair_frag), s)
    repacked = {_frag_base(s.frag) for s in stmts if type(s).__name__ == "FragmentRepack"}
    mmas = [s for s in stmts if type(s).__name__ == "MmaSyncPtx"]
    qk = [s for s in mmas if _frag_base(s.a_frag) not in repacked]
    pv = [s for s in mmas if _frag_base(s.a_frag) in repacked]
    if not qk or not pv:
        raise NotImplementedError("attention needs a score MMA and a PV MMA")
    # the key-chunk loop: the loop that holds the row reductions
    ck = None
    for s in stmts:
        if type(s).__name__ in ("Loop", "StridedLoop") and \
                any(type(x).__name__ == "FragmentRowReduce" for x in _walk(s.body)):
            ck = s.axis.name
            break
    # operands read straight from global memory, or staged through shared memory by
    # cp.async (the staging copy inside the key loop names the global buffer and index)
    copies = {}
    for s in stmts:
        if type(s).__name__ == "CpAsyncCopy":
            copies.setdefault(s.smem, []).append(s)

    def source(ld):
        if ld.src_buffer in spec.buffers:
            return ld.src_buffer, ld.src_index
        cps = copies.get(ld.src_buffer)
        if not cps or len({c.src for c in cps}) != 1 or cps[0].src not in spec.buffers:
            raise NotImplementedError(f"attention operand {ld.src_buffer} not traceable to a buffer")
        for c in cps:
            if any(ck in expr_vars(e) for e in c.src_index):
                return c.src, c.src_index
        return cps[0].src, cps[0].src_index

    q_name, _ = source(frag_src[_frag_base(qk[0].a_frag)])
    k_name, k_index = source(frag_src[_frag_base(qk[0].b_frag)])
    v_name, _ = source(frag_src[_frag_base(pv[0].b_frag)])
    Q, K, V = spec.param(q_name), spec.param(k_name), spec.param(v_name)
    stores = [s for s in stmts if type(s).__name__ == "RegStore"]
    O = spec.param(stores[0].dst_buffer)
    if len({Q.dtype, K.dtype, V.dtype, O.dtype}) != 1:
        raise NotImplementedError("mixed attention dtypes")
    kdims = [i for i, e in enumerate(k_index) if ck in expr_vars(e)]
    if len(kdims) != 1:
        raise NotImplementedError("key axis of K not identifiable")
    kt_layout = kdims[0] == len(K.shape) - 1
    Sq, D = Q.shape[-2], Q.shape[-1]
    Sk = K.shape[-1] if kt_layout else K.shape[-2]
    if (K.shape[-2] if kt_layout else K.shape[-1]) != D or tuple(V.shape[-2:]) != (Sk, D) \
            or tuple(O.shape[-2:]) != (Sq, D):
        raise NotImplementedError("attention operand shapes")
    BH = math.prod(Q.shape[:-2]) if len(Q.shape) > 2 else 1
    for X in (K, V, O):
        if (math.prod(X.shape[:-2]) if len(X.shape) > 2 else 1) != BH:
            raise NotImplementedError("grouped / broadcast heads")
    scale, causal = _score_chain(spec, stmts, {_frag_base(s.c_frag) for s in qk})
    return AttnConfig(BH=BH, Sq=Sq, Sk=Sk, D=D, dtype=Q.dtype, kt_layout=kt_layout, scale=scale,
                      causal=causal, name=spec.name, q_param=Q.name, k_param=K.name,
                      v_param=V.name, o_param=O.name, arg_params=arg_params(spec),
                      buffers=tuple(x.name for x in spec.params))


def _constants(spec, stmts) -> dict:
    """Scalar values the body derives from constant buffers and literals (``Load`` of a
    constant, ``Let`` of a literal, reciprocal / multiply / divide / copy of those)."""
    env = {}
    for s in stmts:
        k = type(s).__name__
        if k == "Load" and s.input in spec.constants and len(s.names) == 1:
            env[s.names[0]] = float(spec.constants[s.input])
        elif k == "Let" and type(s.value).__name__ == "Literal":
            env[s.name] = float(s.value.value)
        elif k == "Assign" and all(a in env for a in s.args):
            a = [env[x] for x in s.args]
            op = s.op.name
            if op == "reciprocal":
                env[s.name] = 1.0 / a[0]
            elif op == "multiply":
                env[s.name] = a[0] * a[1]
            elif op == "divide":
                env[s.name] = a[0] / a[1]
            elif op == "copy":
                env[s.name] = a[0]
    return env


def _is_causal_cond(cond) -> bool:
    """``__frow < __fcol`` (or ``__fcol > __frow``): the query row is before the key."""
    if type(cond).__name__ != "BinaryExpr":
        return False
    names = tuple(getattr(x, "name", None) for x in (cond.left, cond.right))
    return (cond.op == "<" and names == ("__frow", "__fcol")) or \
        (cond.op == ">" and names == ("__fcol", "__frow"))


def _score_chain(spec, stmts, score_frags) -> tuple[float, bool]:
    """Follow one score fragment from the QK MMA to the row-max subtraction and
    return (scale, causal).  Accepted on the way (the reference's ``FragmentApply``
    forms, ``compiler/mma.py:385-437``): copies; multiplies / divides by a constant
    (the softmax scale); adds / subtracts of a constant (a uniform shift, which the
    softmax cancels); ``where(__frow < __fcol, fill, s)`` with a very negative fill
    (the causal mask).  Anything else raises ``NotImplementedError``."""
    env = _constants(spec, stmts)
    applies = [s for s in stmts if type(s).__name__ == "FragmentApply"]

    def frag_args(s):
        return [a for a, kd in zip(s.args, s.kinds) if kd == "frag"]

    start = next((i for i, s in enumerate(applies)
                  if frag_args(s) and _frag_base(frag_args(s)[0]) in score_frags), None)
    if start is None:
        raise NotImplementedError("score fragment never reaches the softmax")
    scale, causal, i = 1.0, False, start
    for _ in range(len(applies)):
        cur = applies[i]
        op, kinds = cur.op.name, tuple(cur.kinds)
        if cur.post:
            raise NotImplementedError("score operation with a post-op")
        unis = [a for a, kd in zip(cur.args, kinds) if kd == "uniform"]
        if op == "copy" and kinds == ("frag",):
            pass
        elif op in ("multiply", "divide") and sorted(kinds) == ["frag", "uniform"] and unis[0] in env:
            if op == "divide" and kinds[0] != "frag":
                raise NotImplementedError("constant divided by the scores")
            v = env[unis[0]]
            scale = scale * v if op == "multiply" else scale / v
        elif op in ("add", "subtract") and sorted(kinds) == ["frag", "uniform"] and \
                (op == "add" or kinds[0] == "frag"):
            pass                               # a uniform shift: the softmax cancels it
        elif op == "where" and kinds == ("coord", "uniform", "frag") and _is_causal_cond(cur.args[0]) \
                and type(cur.args[1]).__name__ == "Literal" and float(cur.args[1].value) <= -1e4:
            causal = True
        elif op == "subtract" and "row" in kinds:
            return scale, causal               # the row-max subtraction: the scores end here
        else:
            raise NotImplementedError(f"score operation {op}{kinds} before the softmax")
        nxt = next((j for j in range(i + 1, len(applies))
                    if frag_args(applies[j]) and _frag_base(frag_args(applies[j])[0]) == cur.out), None)
        if nxt is None:
            raise NotImplementedError("score chain does not reach the row maximum")
        i = nxt
    raise NotImplementedError("score chain does not reach the row maximum")


def analyze_simt(spec) -> AttnConfig:
    """Emmy's SIMT attention form: one cooperative tile per (head, query row, output
    column) streams the keys, ``s = (q . k) * scale [+ mask[row, key]]`` over an inner
    head-dim loop, and keeps an online softmax (running max, rescaled sums) of ``v``
    (the reference lowers it statement by statement, ``compiler/stmts.py``; fixture
    ``x_h_sdpa_mask``: sdpa with an additive ``attn_mask``).  Recognised strictly by its
    index variables and its score chain; anything else raises ``NotImplementedError``."""
    from ..stmts import expr_vars
    if len(spec.body) != 1 or type(spec.body[0]).__name__ != "Tile":
        raise NotImplementedError("not a single-tile kernel")
    tile = spec.body[0]
    loops = [x for x in tile.body if type(x).__name__ in ("Loop", "StridedLoop")]
    if len(loops) != 1:
        raise NotImplementedError("not a key-streaming attention")
    kl = loops[0]
    kv = kl.axis.name
    inner = [x for x in kl.body if type(x).__name__ in ("Loop", "StridedLoop")]
    if not inner:
        raise NotImplementedError("no head-dim loop")
    # emmy may unroll the key step (keys kv, kv + 32, ... each with its own softmax state,
    # combined after the loop: ``x_h_attn_mask``): every replica has the same dot product,
    # and the first one's statements are the score chain
    sig0 = [(type(x).__name__, getattr(getattr(x, "op", None), "name", None)) for x in inner[0].body]
    for other in inner[1:]:
        if [(type(x).__name__, getattr(getattr(x, "op", None), "name", None)) for x in other.body] != sig0 \
                or int(other.axis.extent.value) != int(inner[0].axis.extent.value):
            raise NotImplementedError("unrolled key steps that differ")
    dv = inner[0].axis.name
    body_in = list(inner[0].body)
    loads_in = {x.names[0]: x for x in body_in if type(x).__name__ == "Load" and len(x.names) == 1}
    prods = [x for x in body_in if type(x).__name__ == "Assign" and x.op.name == "multiply"]
    accs = [x for x in body_in if type(x).__name__ == "Accum" and x.op.name == "add"]
    if len(prods) != 1 or len(accs) != 1 or accs[0].value != prods[0].name or \
            len(body_in) != 4 or set(prods[0].args) != set(loads_in):
        raise NotImplementedError("head-dim loop is not a dot product")
    acc = accs[0].name

    def ivars(ld):
        return [expr_vars(e) for e in ld.index]

    q_ld = [x for x in loads_in.values() if not any(kv in v for v in ivars(x))]
    k_ld = [x for x in loads_in.values() if any(kv in v for v in ivars(x))]
    if len(q_ld) != 1 or len(k_ld) != 1:
        raise NotImplementedError("dot product is not query x key")
    q_ld, k_ld = q_ld[0], k_ld[0]
    qi = ivars(q_ld)
    if qi[-1] != {dv} or len(qi[-2]) != 1:
        raise NotImplementedError("query operand layout")
    qvar = next(iter(qi[-2]))
    ki = ivars(k_ld)
    if ki[-2:] == [{kv}, {dv}]:
        kt_layout = False
    elif ki[-2:] == [{dv}, {kv}]:
        kt_layout = True
    else:
        raise NotImplementedError("key operand layout")
    env = _constants(spec, list(_walk(spec.body)))
    stm = list(kl.body)
    if len(inner) > 1:
        stm = stm[:next(i for i, x in enumerate(stm) if x is inner[1])]
    # the dot product may be rounded first (``f16 v4 = copy(acc0)``)
    src = acc
    while True:
        cps = [x for x in stm if type(x).__name__ == "Assign" and x.op.name == "copy" and tuple(x.args) == (src,)]
        if len(cps) != 1:
            break
        src = cps[0].name
    scaled = [x for x in stm if type(x).__name__ == "Assign" and src in x.args]
    if len(scaled) != 1 or scaled[0].op.name != "multiply" or \
            not all(a == src or a in env for a in scaled[0].args):
        raise NotImplementedError("score is not a scaled dot product")
    scale = math.prod(env[a] for a in scaled[0].args if a != src)
    score = scaled[0].name
    loads = {x.names[0]: x for x in stm if type(x).__name__ == "Load" and len(x.names) == 1}
    mask_ld = None
    adds = [x for x in stm if type(x).__name__ == "Assign" and x.op.name == "add" and score in x.args]
    if adds:
        other = [a for a in adds[0].args if a != score]
        if len(adds) != 1 or len(other) != 1 or other[0] not in loads:
            raise NotImplementedError("score shifted by something other than a mask")
        mask_ld = loads[other[0]]
        mi = ivars(mask_ld)
        if mi[-2:] != [{qvar}, {kv}]:
            raise NotImplementedError("mask not indexed by (query, key)")
        score = adds[0].name
    # the running maximum is taken over exactly this score, and the softmax uses exp
    maxes = [x for x in stm if type(x).__name__ == "Accum" and x.op.name == "maximum"]
    if len(maxes) != 1 or maxes[0].value != score or \
            not any(type(x).__name__ == "Assign" and x.op.name == "exp" for x in stm):
        raise NotImplementedError("no online softmax over the score")
    v_ld = [x for x in loads.values() if x is not mask_ld and any(kv in v for v in ivars(x))]
    if len(v_ld) != 1:
        raise NotImplementedError("value operand not identifiable")
    vi = ivars(v_ld[0])
    if vi[-2] != {kv} or len(vi[-1]) != 1:
        raise NotImplementedError("value operand layout")
    dout = next(iter(vi[-1]))
    writes = [x for x in _walk(tile.body) if type(x).__name__ == "Write" and x.output in spec.buffers]
    if len(writes) != 1 or [expr_vars(e) for e in writes[0].index][-2:] != [{qvar}, {dout}]:
        raise NotImplementedError("output not written per (query, column)")
    Q, K, V = spec.param(q_ld.input), spec.param(k_ld.input), spec.param(v_ld[0].input)
    O = spec.param(writes[0].output)
    if len({Q.dtype, K.dtype, V.dtype, O.dtype}) != 1:
        raise NotImplementedError("mixed attention dtypes")
    Sq, D = Q.shape[-2], Q.shape[-1]
    Sk = K.shape[-1] if kt_layout else K.shape[-2]
    if (K.shape[-2] if kt_layout else K.shape[-1]) != D or tuple(V.shape[-2:]) != (Sk, D) \
            or tuple(O.shape[-2:]) != (Sq, D):
        raise NotImplementedError("attention operand shapes")
    BH = math.prod(Q.shape[:-2]) if len(Q.shape) > 2 else 1
    for X in (K, V, O):
        if (math.prod(X.shape[:-2]) if len(X.shape) > 2 else 1) != BH:
            raise NotImplementedError("grouped / broadcast heads")
    extra = {}
    if mask_ld is not None:
        M = spec.param(mask_ld.input)
        if tuple(M.shape[-2:]) != (Sq, Sk):
            raise NotImplementedError("mask shape")
        lead = math.prod(M.shape[:-2]) if len(M.shape) > 2 else 1
        if lead not in (1, BH):
            raise NotImplementedError("mask broadcast over part of the batch x heads")
        extra = dict(mask_param=M.name, mask_dtype=M.dtype, mask_bh_stride=0 if lead == 1 else Sq * Sk)
    return AttnConfig(BH=BH, Sq=Sq, Sk=Sk, D=D, dtype=Q.dtype, kt_layout=kt_layout, scale=scale,
                      name=spec.name, q_param=Q.name, k_param=K.name, v_param=V.name, o_param=O.name,
                      arg_params=arg_params(spec), buffers=tuple(x.name for x in spec.params), **extra)


_DT_REPR = {"f32": "DataType(name='f32', np=dtype('float32'), nbytes=4)",
            "f16": "DataType(name='f16', np=dtype('float16'), nbytes=2)",
            "bf16": "DataType(name='bf16', np=dtype('uint16'), nbytes=2)"}


def score_input_spec(spec):
    """``softmax(S) @ V`` with the scores an input buffer (``tests/problems/x_h_softmax_mm``:
    emmy's tensor-core form reads each score fragment from global memory,
    ``FragmentApply(_s += s[__frow, __fcol])``, and has only the P V MMA).  Returned as an
    element-map kernel over (row, column) of O with the same arithmetic: the row maximum,
    the f32 sum of exp(s - max), P rounded to the operands' 16-bit type times V summed in
    f32 (the MMA's exact products), and O = acc * (1 / l) rounded on the store."""
    from dataclasses import replace
    from ..ir import parse_stmt
    stmts = list(_walk(spec.body))
    gm = [x for x in stmts if type(x).__name__ == "FragmentApply" and "gmem" in (x.kinds or ())]
    if not gm or not any(type(x).__name__ == "FragmentRowReduce" for x in stmts):
        raise NotImplementedError("no score fragment read from memory")
    srcs = {x.args[list(x.kinds).index("gmem")][0] for x in gm}
    if len(srcs) != 1 or any(x.op.name != "add" or x.args[0] != x.out for x in gm):
        raise NotImplementedError("scores other than one input buffer")
    sname = next(iter(srcs))
    staged = {x.smem: x.src for x in stmts if type(x).__name__ == "CpAsyncCopy"}
    bsrc = {staged.get(x.src_buffer, x.src_buffer) for x in stmts
            if type(x).__name__ == "LdmatrixLoad" and x.role == "b"}
    stores = {x.dst_buffer for x in stmts if type(x).__name__ == "RegStore"}
    # the score fragments see nothing but the input, the softmax and (odd sizes) the mask of
    # the tile's padding past the last key, where(__fcol >= Sk, -1e30, s)
    S = spec.param(sname)
    tail = [x for x in stmts if type(x).__name__ == "FragmentApply" and x.op.name == "where"]
    for x in tail:
        c = x.args[0]
        if not (type(c).__name__ == "BinaryExpr" and c.op == ">=" and getattr(c.left, "name", None) == "__fcol"
                and type(c.right).__name__ == "Literal" and int(c.right.value) == S.shape[-1]):
            raise NotImplementedError("a score mask other than the padding past the last key")
    ops = {x.op.name for x in stmts if type(x).__name__ == "FragmentApply" and "gmem" not in (x.kinds or ())
           and x.op.name != "where"}
    if len(bsrc) != 1 or len(stores) != 1 or not ops <= {"subtract", "exp", "multiply"}:
        raise NotImplementedError("not softmax(S) @ V")
    V, O = spec.param(next(iter(bsrc))), spec.param(next(iter(stores)))
    if len(S.shape) != 2 or len(V.shape) != 2 or tuple(O.shape) != (S.shape[0], V.shape[1]) or \
            V.shape[0] != S.shape[1] or V.dtype not in ("f16", "bf16") or O.dtype not in ("f16", "bf16"):
        raise NotImplementedError("softmax(S) @ V shapes / types")
    Sq, Sk, D = S.shape[0], S.shape[1], V.shape[1]
    f32, pdt, odt = _DT_REPR["f32"], _DT_REPR[V.dtype], _DT_REPR[O.dtype]

    def loop(k, body):
        return (f"Loop(axis=Axis(name='{k}', extent=Dim({Sk}), window=None), body=({body}), "
                f"unroll=False, seed=True)")
    ld_s = "Load(names=('{n}',), input='" + sname + "', index=(Var(name='i'), Var(name='{k}')), dtype=None)"
    body = ", ".join([
        loop("k0", ld_s.format(n="s0", k="k0") + ", "
             f"Accum(name='m', value='s0', op=ElementwiseImpl('maximum'), dtype={f32}, axes=('k0',), base=None)"),
        loop("k1", ld_s.format(n="s1", k="k1") + ", "
             f"Assign(name='d1', op=ElementwiseImpl('subtract'), args=('s1', 'm'), dtype={f32}), "
             f"Assign(name='e1', op=ElementwiseImpl('exp'), args=('d1',), dtype={f32}), "
             f"Accum(name='l', value='e1', op=ElementwiseImpl('add'), dtype={f32}, axes=('k1',), base=None)"),
        loop("k2", ld_s.format(n="s2", k="k2") + ", "
             f"Assign(name='d2', op=ElementwiseImpl('subtract'), args=('s2', 'm'), dtype={f32}), "
             f"Assign(name='e2', op=ElementwiseImpl('exp'), args=('d2',), dtype={f32}), "
             f"Assign(name='p2', op=ElementwiseImpl('copy'), args=('e2',), dtype={pdt}), "
             f"Load(names=('v2',), input='{V.name}', index=(Var(name='k2'), Var(name='c')), dtype=None), "
             f"Assign(name='t2', op=ElementwiseImpl('multiply'), args=('p2', 'v2'), dtype={f32}), "
             f"Accum(name='acc', value='t2', op=ElementwiseImpl('add'), dtype={f32}, axes=('k2',), base=None)"),
        f"Assign(name='rl', op=ElementwiseImpl('reciprocal'), args=('l',), dtype={f32})",
        f"Assign(name='r', op=ElementwiseImpl('multiply'), args=('acc', 'rl'), dtype={f32})",
        f"Write(output='{O.name}', index=(Var(name='i'), Var(name='c')), values=('r',), value_dtype={odt}, "
        f"atomic=False, swizzle='NONE')",
    ])
    tile = parse_stmt(f"Tile(axes=(Axis(name='i', extent=Dim({Sq}), window=None), "
                      f"Axis(name='c', extent=Dim({D}), window=None)), body=({body},), block_threads=256, "
                      f"aux_threads=0, raster_axes=None, raster_group=None, raster_orient='m')")
    return replace(spec, body=(tile,))


def emit_attention(spec) -> str:
    try:
        cfg = analyze(spec)
    except NotImplementedError:
        # softmax(S) @ V over an input S: an element map of the same arithmetic
        from .pointwise import emit_map
        return emit_map(score_input_spec(spec))
    return emit_attention_module(cfg)
