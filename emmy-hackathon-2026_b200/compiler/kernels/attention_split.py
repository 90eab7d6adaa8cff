"""Persistent split-key attention for unmasked, non-causal O = softmax(Q K^T * scale) V.

The same operation as ``attention.py``'s two-tile template (which serves every
attention problem by default, causal, masked, ragged and pre-transposed-K ones
included); selected with ``AttnConfig.schedule = "split_keys"``.  It schedules the work
so that the next block's scores never wait for the current block's probabilities:

* one query tile of 128 rows at a time; the CTA is persistent and walks the tiles
  ``ctaid, ctaid + grid, ...`` (tile -> batch x head ``tile / (Sq / 128)``, query rows
  ``128 * (tile % (Sq / 128))``), so one tile's epilogue overlaps the next tile's first
  scores and the K / V stream never drains between tiles;
* TMEM (512 columns): two S buffers of 128 columns, S(g) in buffer g % 2 for the g-th
  key block the CTA processes; two O accumulators of 128 columns, O_h for the keys of
  half h of every block;
* two softmax warpgroups, one per 64-key half of every 128-key block: warpgroup h
  (warps 4h .. 4h+3) thread r owns query row r of keys [64h, 64h + 64).  Each half keeps
  its own running maximum m_h and row sum l_h (lazy rescale of its own O_h past 2^8),
  so the two warpgroups never exchange anything inside a tile; P_h (bf16 / f16 pairs)
  goes back into columns [64h, 64h + 32) of the S buffer, where the PV MMA reads it.
  The exponentials take turns on the MUFU pipe (``turn`` barriers: half 0 of block g,
  then half 1 of block g, then half 0 of block g + 1 ...), so one half's exponentials
  overlap the other half's loads, maxima and stores;
* epilogue, once per tile: each half waits for its own last product, the halves trade
  (m_h, l_h) through shared memory, and row r of O is
  ``(O_0 2^(m_0 - M) + O_1 2^(m_1 - M)) / (l_0 2^(m_0 - M) + l_1 2^(m_1 - M))`` with
  ``M = max(m_0, m_1)``; warpgroup h writes head dims [64h, 64h + 64);
* control warpgroup: warp 8 lane 0 issues TMA (Q tiles double-buffered, K and V through
  rings of two slots each, in the order the MMA streams consume them: V(g) then
  K(g + 2)); warp 9 allocates TMEM; lane 0 of warp 9 + h issues half h's stream:
  ``S_h(0)``, ``S_h(1)``, then per block ``O_h += P_h(g) V_g`` and ``S_h(g + 2) = Q K_{g+2}[64h ..]^T``
  (M = 128, N = 64).  One thread's tcgen05 operations complete in issue order, so
  ``S_h(g + 2)`` overwrites the columns of ``P_h(g)`` only after the product that reads
  them, and each half's chain (softmax -> PV -> next scores) is independent of the
  other's.

Per block the MMA threads wait for V(g), P_h(g) and K(g + 2) and commit twice
(``o_done[h]``: O_h holds block g; ``s_full[h]``: S_h ready).  The producer reuses a K
slot once both halves' ``s_full`` and a V slot once both halves' ``o_done`` completed,
so the ring needs no empty barriers of its own; the shared-memory descriptors of the
ring slots are formed once and a K step adds its offset to the 64-bit descriptor.
The protocol is checked under random schedules by ``tests/test_attention_split_protocol.py``.

Measured on the B200 (BASELINE 8 x 32 x 4096 x 128, bench.py): 0.87-0.91x the two-tile
template.  The per-half score products are M = 128, N = 64 MMAs, which cost about as much
per instruction as N = 128 ones (~85 clocks each in %clock64 stamps of the MMA threads),
so a block takes 24 MMA instructions (~2050 clocks) where the template needs 16 per tile
and block; shared-memory bank reads stay low (14 % of peak), so that is not the limit.

Every mbarrier wait is bounded (``tc.Waits``); a wait that gives up raises the CTA's
abort flag and every role leaves through the common exit, which frees TMEM.
"""

from __future__ import annotations

from ..ptx import Ptx, entry, f32_hex, module
from .attention import AB_FORMAT, LOG2E, RESCALE_LOG2, AttnConfig, _max_tree, emit_exp2_poly
from .common import load_pointer, param_symbol
from .gemm import SMS
from .tc import Waits, instr_desc, smem_desc_hi, smem_desc_lo_const

SLOT = 128 * 128 * 2                 # one Q, K or V tile: 128 rows x 128 head dims, 16-bit
Q_OFF, K_OFF, V_OFF = 0, 2 * SLOT, 4 * SLOT
X_OFF = 6 * SLOT                     # (m, l) exchange: [tile parity][half][row] x 8 bytes
T_OFF = X_OFF + 2 * 2 * 128 * 8      # block row sums handed over with the MUFU turn: [half][row]
SMEM = T_OFF + 2 * 128 * 4 + 1024
NTHREADS = 384

# mbarriers (8 bytes each): name -> (offset, count, arrivals)
# (a K slot is free again once S of its block is done: s_full; a V slot once O += P V of
# its block is done: o_done -- the ring needs no empty barriers of its own)
# s_full, p_ready, o_done: [half][buffer g % 2]; q_empty takes both halves' last S
_BARS = [("q_full", 2, 1), ("q_empty", 2, 2), ("k_full", 2, 1), ("v_full", 2, 1),
         ("s_full", 4, 1), ("p_ready", 4, 128), ("o_done", 4, 1), ("o_free", 1, 256), ("xch", 2, 256),
         ("turn", 2, 128)]
BAR = {}
_o = 0
for _n, _c, _a in _BARS:
    BAR[_n] = _o
    _o += 8 * _c
NBAR = _o // 8


def eligible(cfg: AttnConfig) -> bool:
    """The problems this kernel serves: every (query, key) pair takes part, whole 128-row
    query tiles and 128-key blocks, head dim 128, K in [.., Sk, D] rows."""
    return (not cfg.causal and cfg.mask_param is None and not cfg.kt_layout and cfg.p_tmem
            and cfg.D == 128 and cfg.dtype in AB_FORMAT and cfg.scale > 0
            and cfg.Sq % 128 == 0 and cfg.Sk % 128 == 0 and cfg.Sk >= 256
            and (cfg.kv_group == 1 or (cfg.heads and cfg.heads % cfg.kv_group == 0
                                       and cfg.BH % cfg.heads == 0)))


def emit_attention_split_module(cfg: AttnConfig, sms: int = SMS) -> str:
    if not eligible(cfg):
        raise NotImplementedError("split-key attention: unsupported problem")
    p = Ptx()
    nq = cfg.Sq // 128                   # query tiles per batch x head
    nblk = cfg.Sk // 128                 # key blocks per tile
    ntiles = cfg.BH * nq
    grid = min(sms, ntiles)
    fmt = AB_FORMAT[cfg.dtype]
    idesc_qk64 = instr_desc(128, 64, fmt, fmt, False, False)
    idesc_pv = instr_desc(128, 128, fmt, fmt, False, True)
    sw_hi = smem_desc_hi(1024)
    kmaj_lo = smem_desc_lo_const(16)
    v_lo = smem_desc_lo_const(128 * 128)
    scale_log2 = cfg.scale * LOG2E

    p.comment(f"split-key persistent tcgen05 attention BH={cfg.BH} Sq={cfg.Sq} Sk={cfg.Sk} "
              f"D={cfg.D} {cfg.dtype}, {ntiles} query tiles over {grid} CTAs, {nblk} key blocks")
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
    p0 = p.reg("pred")
    l_init = p.label("init_done")
    p.emit(f"setp.ne.u32 {p0}, {tid}, 0\n@{p0} bra {l_init}")
    for n, c, a in _BARS:
        for i in range(c):
            p.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{BAR[n] + 8 * i}], {a}")
    p.emit(f"st.shared.u32 [{abort}], 0\nfence.mbarrier_init.release.cluster\nfence.proxy.async.shared::cta")
    p.place(l_init)
    W_TMA, W_MMA, W_S = 8, 9, 10
    p1 = p.reg("pred")
    l_alloc = p.label("alloc_done")
    p.emit(f"setp.ne.u32 {p1}, {warp}, {W_MMA}\n@{p1} bra {l_alloc}")
    p.emit(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], 512\n"
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
    # this CTA's tiles and key blocks: ntile = (ntiles - 1 - ctaid) / grid + 1
    cta, ntile, total = p.regs("u32", 3)
    p.emit(f"""
        mov.u32 {cta}, %ctaid.x
        sub.u32 {ntile}, {ntiles - 1}, {cta}
        div.u32 {ntile}, {ntile}, {grid}
        add.u32 {ntile}, {ntile}, 1
        mul.lo.u32 {total}, {ntile}, {nblk}
    """)

    def bar(name, idx=None):
        """Address of barrier ``name`` (+ 8 * idx for a register index)."""
        r = p.reg("u32")
        if idx is None:
            p.emit(f"add.u32 {r}, {bars}, {BAR[name]}")
        else:
            p.emit(f"mad.lo.u32 {r}, {idx}, 8, {bars}\nadd.u32 {r}, {r}, {BAR[name]}")
        return r

    def bar_hs(name, h, sl):
        """Address of [half h][buffer sl] of a barrier pair array (h a constant)."""
        r = p.reg("u32")
        p.emit(f"mad.lo.u32 {r}, {sl}, 8, {bars}\nadd.u32 {r}, {r}, {BAR[name] + 16 * h}")
        return r

    def bit(x, k):
        """(x >> k) & 1 in a fresh register."""
        r = p.reg("u32")
        p.emit(f"bfe.u32 {r}, {x}, {k}, 1")
        return r

    def tile_of(it):
        """(batch x head, first query row) of this CTA's it-th tile."""
        t, bh, q0 = p.regs("u32", 3)
        p.emit(f"""
            mad.lo.u32 {t}, {it}, {grid}, {cta}
            div.u32 {bh}, {t}, {nq}
            rem.u32 {q0}, {t}, {nq}
            shl.b32 {q0}, {q0}, 7
        """)
        return bh, q0

    def kv_head(bh):
        if cfg.kv_group == 1:
            return bh
        kvbh, hq = p.reg("u32"), p.reg("u32")
        p.emit(f"div.u32 {kvbh}, {bh}, {cfg.heads}\nrem.u32 {hq}, {bh}, {cfg.heads}\n"
               f"div.u32 {hq}, {hq}, {cfg.kv_group}\nmad.lo.u32 {kvbh}, {kvbh}, {cfg.heads // cfg.kv_group}, {hq}")
        return kvbh

    class Cursor:
        """(g, j, it): the CTA's g-th key block is block j of its it-th tile."""

        def __init__(self):
            self.g, self.j, self.it = p.regs("u32", 3)
            p.emit(f"mov.u32 {self.g}, 0\nmov.u32 {self.j}, 0\nmov.u32 {self.it}, 0")

        def advance(self):
            pw = p.reg("pred")
            p.emit(f"""
                add.u32 {self.g}, {self.g}, 1
                add.u32 {self.j}, {self.j}, 1
                setp.eq.u32 {pw}, {self.j}, {nblk}
                @{pw} mov.u32 {self.j}, 0
                @{pw} add.u32 {self.it}, {self.it}, 1
            """)

    # -------------------------------------------------------------- role dispatch
    l_ctl, l_soft = p.label("role_control"), p.label("role_softmax")
    pc = p.reg("pred")
    p.emit(f"setp.lt.u32 {pc}, {warp}, 8\n@{pc} bra {l_soft}")
    p.place(l_ctl)
    l_mma = p.label("role_mma")
    pr, pl = p.reg("pred"), p.reg("pred")
    p.emit(f"setp.ne.u32 {pr}, {warp}, {W_TMA}\n@{pr} bra {l_mma}\nsetp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")

    # ------------------------------------------------------------------ producer
    p.emit(f"prefetch.tensormap [{tq}]\nprefetch.tensormap [{tk}]\nprefetch.tensormap [{tv}]")

    def tma_tile(tmap, dst0, row0, head, fb):
        for db in range(2):
            dst = p.reg("u32")
            p.emit(f"add.u32 {dst}, {dst0}, {db * 16384}")
            p.emit(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                   f"[{dst}], [{tmap}, {{{db * 64}, {row0}, {head}}}], [{fb}]")

    def empty_wait(name, g, full_name, halves=False):
        """Wait until slot g % 2 of a two-slot ring is free (``name`` -- for both halves,
        when ``halves`` -- completed for the slot's previous use, g - 2); returns (full
        barrier, slot)."""
        sl = bit(g, 0)
        par = bit(g, 1)
        p.emit(f"xor.b32 {par}, {par}, 1")
        for h in (range(2) if halves else ()):
            waits.wait(bar_hs(name, h, sl), par, "producer", finish)
        if not halves:
            waits.wait(bar(name, sl), par, "producer", finish)
        fb = bar(full_name, sl)
        p.emit(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {SLOT}")
        return fb, sl

    def load_k(c):
        bh, q0 = tile_of(c.it)
        kvbh = kv_head(bh)
        l_noq = p.label("p_noq")
        pq = p.reg("pred")
        p.emit(f"setp.ne.u32 {pq}, {c.j}, 0\n@{pq} bra {l_noq}")
        fq, sq = empty_wait("q_empty", c.it, "q_full")
        dq = p.reg("u32")
        p.emit(f"mad.lo.u32 {dq}, {sq}, {SLOT}, {base}\nadd.u32 {dq}, {dq}, {Q_OFF}")
        tma_tile(tq, dq, q0, bh, fq)
        p.place(l_noq)
        fk, sk = empty_wait("s_full", c.g, "k_full", halves=True)
        dk, key0 = p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {dk}, {sk}, {SLOT}, {base}\nadd.u32 {dk}, {dk}, {K_OFF}\nshl.b32 {key0}, {c.j}, 7")
        tma_tile(tk, dk, key0, kvbh, fk)

    def load_v(c):
        bh, _ = tile_of(c.it)
        kvbh = kv_head(bh)
        fv, sv = empty_wait("o_done", c.g, "v_full", halves=True)
        dv, key0 = p.reg("u32"), p.reg("u32")
        p.emit(f"mad.lo.u32 {dv}, {sv}, {SLOT}, {base}\nadd.u32 {dv}, {dv}, {V_OFF}\nshl.b32 {key0}, {c.j}, 7")
        tma_tile(tv, dv, key0, kvbh, fv)

    ck, cv = Cursor(), Cursor()
    load_k(ck)
    ck.advance()
    load_k(ck)
    ck.advance()
    l_pl = p.label("p_loop")
    p.place(l_pl)
    load_v(cv)
    cv.advance()
    l_nok = p.label("p_nok")
    pk = p.reg("pred")
    p.emit(f"setp.ge.u32 {pk}, {ck.g}, {total}\n@{pk} bra {l_nok}")
    load_k(ck)
    ck.advance()
    p.place(l_nok)
    pv_ = p.reg("pred")
    p.emit(f"setp.lt.u32 {pv_}, {cv.g}, {total}\n@{pv_} bra {l_pl}\nbra {finish}")

    # ----------------------------------------------------------------------- MMA
    p.place(l_mma)
    p.emit(f"setp.gt.u32 {pr}, {warp}, {W_S}\n@{pr} bra {finish}\nsetp.ne.u32 {pl}, {lane}, 0\n@{pl} bra {finish}")

    def commit(addr):
        p.emit(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{addr}]")

    def full_wait(name, idx, par):
        waits.wait(bar(name, idx), par, "mma", finish)
        p.emit("tcgen05.fence::after_thread_sync")

    # descriptor low words of slot 0 of the Q, K and V rings; slot s is 2048 (SLOT >> 4)
    # further, and a K step inside a tile adds its byte offset >> 4 to the 64-bit
    # descriptor (start addresses stay below 2^18 bytes, so the field never carries)
    lo0 = {}
    for name, off, lbo in (("q", Q_OFF, kmaj_lo), ("k", K_OFF, kmaj_lo), ("v", V_OFF, v_lo)):
        r = p.reg("u32")
        p.emit(f"add.u32 {r}, {base}, {off}\nshr.u32 {r}, {r}, 4\nor.b32 {r}, {r}, {lbo}")
        lo0[name] = r

    def slot_desc(name, sl):
        lo, d = p.reg("u32"), p.reg("b64")
        p.emit(f"mad.lo.u32 {lo}, {sl}, {SLOT >> 4}, {lo0[name]}\nmov.b64 {d}, {{{lo}, {sw_hi}}}")
        return d

    o_t = [p.reg("u32") for _ in range(2)]
    for h in range(2):
        p.emit(f"add.u32 {o_t[h]}, {tbase}, {256 + 128 * h}")

    def issue_s(c, h):
        """S_h(g) = Q K_g[keys 64h .. 64h + 63]^T into columns [64h, 64h + 64) of S
        buffer g % 2 (M = 128, N = 64)."""
        sl, qs = bit(c.g, 0), bit(c.it, 0)
        l_qok = p.label("m_qok")
        pq = p.reg("pred")
        p.emit(f"setp.ne.u32 {pq}, {c.j}, 0\n@{pq} bra {l_qok}")
        full_wait("q_full", qs, bit(c.it, 1))
        p.place(l_qok)
        full_wait("k_full", sl, bit(c.g, 1))
        dq, dk = slot_desc("q", qs), slot_desc("k", sl)
        st = p.reg("u32")
        p.emit(f"mad.lo.u32 {st}, {sl}, 128, {tbase}\nadd.u32 {st}, {st}, {64 * h}")
        for kk in range(8):
            off = ((kk // 4) * 16384 + (kk % 4) * 32) >> 4
            koff = off + ((64 * h * 128) >> 4)      # key rows 64h.. of the 128-byte-row box
            qd, kd = p.reg("b64"), p.reg("b64")
            p.emit(f"add.s64 {qd}, {dq}, {off}\nadd.s64 {kd}, {dk}, {koff}")
            pe = pfalse if kk == 0 else ptrue
            p.emit(f"tcgen05.mma.cta_group::1.kind::f16 [{st}], {qd}, {kd}, {idesc_qk64}, {pe}")
        # S_h(g) complete for softmax half h; with the other half's, K slot g % 2 is free
        commit(bar_hs("s_full", h, sl))
        l_qkeep = p.label("m_qkeep")
        pl_ = p.reg("pred")
        p.emit(f"setp.ne.u32 {pl_}, {c.j}, {nblk - 1}\n@{pl_} bra {l_qkeep}")
        commit(bar("q_empty", qs))
        p.place(l_qkeep)

    def issue_pv(c, h):
        """O_h (+)= P_h(g) V_g[keys 64h .. 64h + 63]."""
        sl, par = bit(c.g, 0), bit(c.g, 1)
        pfirst = p.reg("pred")
        p.emit(f"setp.eq.u32 {pfirst}, {c.j}, 0")
        l_ofree = p.label("m_ofree")
        pn = p.reg("pred")
        p.emit(f"setp.eq.u32 {pn}, {c.it}, 0\nor.pred {pn}, {pn}, !{pfirst}\n@{pn} bra {l_ofree}")
        pit = p.reg("u32")
        p.emit(f"sub.u32 {pit}, {c.it}, 1\nand.b32 {pit}, {pit}, 1")
        full_wait("o_free", None, pit)
        p.place(l_ofree)
        full_wait("v_full", sl, par)
        waits.wait(bar_hs("p_ready", h, sl), par, "mma", finish)
        p.emit("tcgen05.fence::after_thread_sync")
        dv = slot_desc("v", sl)
        pa0 = p.reg("u32")
        p.emit(f"mad.lo.u32 {pa0}, {sl}, 128, {tbase}")
        pe0 = p.reg("pred")
        p.emit(f"not.pred {pe0}, {pfirst}")
        for kk in range(4):
            vd, pa = p.reg("b64"), p.reg("u32")
            p.emit(f"add.s64 {vd}, {dv}, {(4 * h + kk) * 128}\nadd.u32 {pa}, {pa0}, {64 * h + 8 * kk}")
            pe = pe0 if kk == 0 else ptrue
            p.emit(f"tcgen05.mma.cta_group::1.kind::f16 [{o_t[h]}], [{pa}], {vd}, {idesc_pv}, {pe}")
        # O_h holds block g (softmax half h); with the other half's, V slot g % 2 is free
        commit(bar_hs("o_done", h, sl))

    # warp 9 + h, lane 0: half h's stream S_h(0), S_h(1), then O_h += P_h(g) V_g and
    # S_h(g + 2) per block; one thread's tcgen05 operations run in issue order, so
    # S_h(g + 2) overwrites the columns of P_h(g) only after the product that reads them
    l_half1 = p.label("role_half1")
    p.emit(f"setp.ne.u32 {pr}, {warp}, {W_MMA}\n@{pr} bra {l_half1}")
    for h in range(2):
        if h == 1:
            p.place(l_half1)
        cs, cp = Cursor(), Cursor()
        for _ in range(2):
            issue_s(cs, h)
            cs.advance()
        l_ml = p.label("m_loop")
        p.place(l_ml)
        issue_pv(cp, h)
        cp.advance()
        l_nos = p.label("m_nos")
        ps_ = p.reg("pred")
        p.emit(f"setp.ge.u32 {ps_}, {cs.g}, {total}\n@{ps_} bra {l_nos}")
        issue_s(cs, h)
        cs.advance()
        p.place(l_nos)
        pm_ = p.reg("pred")
        p.emit(f"setp.lt.u32 {pm_}, {cp.g}, {total}\n@{pm_} bra {l_ml}\nbra {finish}")

    # ------------------------------------------------------------------ softmax
    p.place(l_soft)
    _emit_softmax_halves(p, cfg, ptr, bars, tbase, base, warp, lane, total, tile_of, bar, bit,
                         Cursor, scale_log2, waits, finish)

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
        tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tbase}, 512
    """)
    p.place(done)
    p.emit("ret")

    params = list(cfg.arg_params or [f".param .u64 {param_symbol(n)}" for n in cfg.buffers])
    params += [".param .align 64 .b8 param__tmap_q[128]", ".param .align 64 .b8 param__tmap_k[128]",
               ".param .align 64 .b8 param__tmap_v[128]", ".param .u64 param__status"]
    cap = 65536 // NTHREADS // 8 * 8
    text = entry(cfg.name, params, p, maxntid=NTHREADS, extra_directives=f"\n.maxnreg {cap}")
    statics = (f"\t.shared .align 8 .b64 gbars[{NBAR}];\n\t.shared .align 4 .u32 gabort;\n"
               f"\t.shared .align 4 .u32 gtmem;\n")
    text = text.replace("{\n", "{\n" + statics, 1)
    eb = 2
    tmap = {"dtype": cfg.dtype, "box": [64, 128, 1], "swizzle": 128}
    launch = {
        "kind": "attention", "grid": [grid, 1, 1], "block": [NTHREADS, 1, 1],
        "cluster": [1, 1, 1], "smem": SMEM, "flops": 4 * cfg.BH * cfg.Sq * cfg.Sk * cfg.D,
        "exps": cfg.BH * cfg.Sq * cfg.Sk, "schedule": "split_keys",
        "extra_params": [
            {"kind": "tmap", "buffer": cfg.q_param, "dims": [cfg.D, cfg.Sq, cfg.BH],
             "strides": [cfg.D * eb, cfg.Sq * cfg.D * eb], **tmap},
            {"kind": "tmap", "buffer": cfg.k_param, "dims": [cfg.D, cfg.Sk, cfg.BHKV],
             "strides": [cfg.D * eb, cfg.Sk * cfg.D * eb], **tmap},
            {"kind": "tmap", "buffer": cfg.v_param, "dims": [cfg.D, cfg.Sk, cfg.BHKV],
             "strides": [cfg.D * eb, cfg.Sk * cfg.D * eb], **tmap},
            {"kind": "status"},
        ],
    }
    return module([text], launch, globals_=[".extern .shared .align 1024 .b8 dsmem[];"])


def _emit_softmax_halves(p: Ptx, cfg: AttnConfig, ptr, bars, tbase, base, warp, lane, total,
                         tile_of, bar, bit, Cursor, scale_log2, waits: Waits, finish) -> None:
    """Warpgroup h = warp / 4, thread = query row 32 (warp % 4) + lane of keys
    [64h, 64h + 64) of every block; the tile's epilogue at its last block."""
    nblk = cfg.Sk // 128
    h, q, row, lanebits = p.regs("u32", 4)
    p.emit(f"""
        shr.u32 {h}, {warp}, 2
        and.b32 {q}, {warp}, 3
        mad.lo.u32 {row}, {q}, 32, {lane}
        shl.b32 {lanebits}, {q}, 21
    """)
    s_half, o_h, o_0, ph0 = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("pred")
    p.emit(f"""
        add.u32 {o_0}, {tbase}, {lanebits}
        mad.lo.u32 {s_half}, {h}, 64, {o_0}
        mad.lo.u32 {o_h}, {h}, 128, {o_0}
        add.u32 {o_h}, {o_h}, 256
        add.u32 {o_0}, {o_0}, 256
        setp.eq.u32 {ph0}, {h}, 0
    """)
    # this row's (m, l) slot in the exchange area and the other half's
    xs, xo = p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {xs}, {h}, 128, {row}
        mad.lo.u32 {xs}, {xs}, 8, {base}
        add.u32 {xs}, {xs}, {X_OFF}
        xor.b32 {xo}, {h}, 1
        mad.lo.u32 {xo}, {xo}, 128, {row}
        mad.lo.u32 {xo}, {xo}, 8, {base}
        add.u32 {xo}, {xo}, {X_OFF}
    """)
    tsum = p.reg("u32")
    p.emit(f"mad.lo.u32 {tsum}, {h}, 128, {row}\nmad.lo.u32 {tsum}, {tsum}, 4, {base}\n"
           f"add.u32 {tsum}, {tsum}, {T_OFF}")
    cvt = "cvt.rn.bf16x2.f32" if cfg.dtype == "bf16" else "cvt.rn.f16x2.f32"
    m, l = p.reg("f32"), p.reg("f32")
    p.emit(f"mov.f32 {m}, 0f00000000\nmov.f32 {l}, 0f00000000")
    slr, sl2 = p.reg("f32"), p.reg("b64")
    p.emit(f"mov.f32 {slr}, {f32_hex(scale_log2)}\nmov.b64 {sl2}, {{{slr}, {slr}}}")
    c = Cursor()
    l_blk = p.label("s_blk")
    p.place(l_blk)
    sl, par = bit(c.g, 0), bit(c.g, 1)
    hs = p.reg("u32")                       # [half][buffer] barrier index h * 2 + g % 2
    p.emit(f"mad.lo.u32 {hs}, {h}, 2, {sl}")
    waits.wait(bar("s_full", hs), par, "softmax", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    sta = p.reg("u32")
    p.emit(f"mad.lo.u32 {sta}, {sl}, 128, {s_half}")
    sv = [p.reg("b32") for _ in range(64)]
    for k in range(2):
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(sv[32 * k:32 * k + 32])}}}, "
               f"[{sta}+{32 * k}]")
    p.emit("tcgen05.wait::ld.sync.aligned")
    fv = [p.reg("f32") for _ in range(64)]
    for i in range(64):
        p.emit(f"mov.b32 {fv[i]}, {sv[i]}")
    mx = p.reg("f32")
    p.emit(f"mul.rn.f32 {mx}, {_max_tree(p, fv)}, {f32_hex(scale_log2)}")
    # running maximum of this half: the block's at a tile's first block, else lazily
    pfirst, prs, pnf = p.reg("pred"), p.reg("pred"), p.reg("pred")
    mn, thr, alpha, d0 = p.regs("f32", 4)
    p.emit(f"""
        setp.eq.u32 {pfirst}, {c.j}, 0
        max.f32 {mn}, {m}, {mx}
        add.rn.f32 {thr}, {m}, {f32_hex(RESCALE_LOG2)}
        setp.gt.f32 {prs}, {mn}, {thr}
        not.pred {pnf}, {pfirst}
        and.pred {prs}, {prs}, {pnf}
        @{pfirst} mov.f32 {m}, {mx}
        @{pfirst} mov.f32 {l}, 0f00000000
        mov.f32 {alpha}, 0f3F800000
        sub.rn.f32 {d0}, {m}, {mn}
        @{prs} ex2.approx.ftz.f32 {alpha}, {d0}
        @{prs} mov.f32 {m}, {mn}
        mul.rn.f32 {l}, {l}, {alpha}
    """)
    pany = p.reg("pred")
    l_nores = p.label("s_nores")
    p.emit(f"vote.sync.any.pred {pany}, {prs}, -1\n@!{pany} bra {l_nores}")
    # O_h *= alpha once O_h += P_h(g - 1) V has landed (o_done[h][(g - 1) % 2], use
    # (g - 1) / 2)
    gm1, oi, opar = p.regs("u32", 3)
    p.emit(f"sub.u32 {gm1}, {c.g}, 1\nand.b32 {oi}, {gm1}, 1\nmad.lo.u32 {oi}, {h}, 2, {oi}\n"
           f"bfe.u32 {opar}, {gm1}, 1, 1")
    waits.wait(bar("o_done", oi), opar, "softmax", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    ov = [p.reg("b32") for _ in range(32)]
    for k in range(4):
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{o_h}+{32 * k}]")
        p.emit("tcgen05.wait::ld.sync.aligned")
        for i in range(32):
            f = p.reg("f32")
            p.emit(f"mov.b32 {f}, {ov[i]}\nmul.rn.f32 {f}, {f}, {alpha}\nmov.b32 {ov[i]}, {f}")
        p.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{o_h}+{32 * k}], {{{', '.join(ov)}}}")
    p.emit("tcgen05.wait::st.sync.aligned")
    p.place(l_nores)
    # the exponentials take turns on the MUFU pipe: half 0 of block g after half 1 of
    # block g - 1 (turn[1], use g - 1), half 1 after half 0 of block g (turn[0], use g),
    # so one half's exponentials overlap the other half's loads, maxima and stores
    l_myturn = p.label("s_myturn")
    pskip, tpar, tbar = p.reg("pred"), p.reg("u32"), p.reg("u32")
    p.emit(f"""
        setp.eq.u32 {pskip}, {c.g}, 0
        and.pred {pskip}, {pskip}, {ph0}
        @{pskip} bra {l_myturn}
        add.u32 {tpar}, {c.g}, 1
        add.u32 {tpar}, {tpar}, {h}
        and.b32 {tpar}, {tpar}, 1
        xor.b32 {tbar}, {h}, 1
    """)
    waits.wait(bar("turn", tbar), tpar, "softmax", finish)
    p.place(l_myturn)
    # p = 2^(s * scale * log2e - m), row sum, pack to 16-bit pairs
    negm, nm2 = p.reg("f32"), p.reg("b64")
    p.emit(f"neg.f32 {negm}, {m}\nmov.b64 {nm2}, {{{negm}, {negm}}}")
    ps = []
    for i in range(0, 64, 2):
        x2, e2 = p.reg("b64"), p.reg("b64")
        ea, eb = p.reg("f32"), p.reg("f32")
        p.emit(f"mov.b64 {x2}, {{{fv[i]}, {fv[i + 1]}}}\n"
               f"fma.rn.f32x2 {e2}, {x2}, {sl2}, {nm2}\nmov.b64 {{{ea}, {eb}}}, {e2}")
        for k, e in ((i, ea), (i + 1, eb)):
            if cfg.poly_every and k % cfg.poly_every == cfg.poly_every - 1:
                emit_exp2_poly(p, e, e)
            else:
                p.emit(f"ex2.approx.ftz.f32 {e}, {e}")
            ps.append(e)
    packed = [p.reg("b32") for _ in range(32)]
    for i in range(32):
        p.emit(f"{cvt} {packed[i]}, {ps[2 * i + 1]}, {ps[2 * i]}")
    red = []
    for i in range(0, 64, 2):
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
    s0, s1 = p.reg("f32"), p.reg("f32")
    p.emit(f"mov.b64 {{{s0}, {s1}}}, {red[0]}\nadd.rn.f32 {s0}, {s0}, {s1}\nadd.rn.f32 {l}, {l}, {s0}")
    # pass the MUFU turn once every exponential of the block is done: the block's row
    # sum (which needs all of them) goes to shared memory ahead of the releasing arrive
    p.emit(f"st.shared.f32 [{tsum}], {s0}")
    p.emit(f"mbarrier.arrive.shared::cta.b64 _, [{bar('turn', h)}]")
    # P_h over the first 32 columns of this half's S columns; hand it to the MMA thread
    p.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{sta}], {{{', '.join(packed)}}}")
    p.emit("tcgen05.wait::st.sync.aligned\ntcgen05.fence::before_thread_sync")
    p.emit(f"mbarrier.arrive.shared::cta.b64 _, [{bar('p_ready', hs)}]")
    l_next = p.label("s_next")
    plast = p.reg("pred")
    p.emit(f"setp.ne.u32 {plast}, {c.j}, {nblk - 1}\n@{plast} bra {l_next}")

    # ------------------------------------------------------------ tile epilogue
    # O_h += P_h(g) V_g landed (o_done[h][g % 2], use g / 2); each half waits for its own
    # before the exchange, so past the exchange both O_0 and O_1 are final
    waits.wait(bar("o_done", hs), par, "softmax", finish)
    tp, xsa, xoa = p.regs("u32", 3)
    p.emit(f"""
        and.b32 {tp}, {c.it}, 1
        mad.lo.u32 {xsa}, {tp}, 2048, {xs}
        mad.lo.u32 {xoa}, {tp}, 2048, {xo}
        st.shared.v2.f32 [{xsa}], {{{m}, {l}}}
    """)
    xb = bar("xch", tp)
    p.emit(f"mbarrier.arrive.shared::cta.b64 _, [{xb}]")
    waits.wait(xb, bit(c.it, 1), "softmax", finish)
    p.emit("bar.warp.sync -1\ntcgen05.fence::after_thread_sync")
    mo, lo, mm, a_s, a_o, ll, inv, c0, c1, cs, co = p.regs("f32", 11)
    p.emit(f"""
        ld.shared.v2.f32 {{{mo}, {lo}}}, [{xoa}]
        max.f32 {mm}, {m}, {mo}
        sub.rn.f32 {a_s}, {m}, {mm}
        ex2.approx.ftz.f32 {a_s}, {a_s}
        sub.rn.f32 {a_o}, {mo}, {mm}
        ex2.approx.ftz.f32 {a_o}, {a_o}
        mul.rn.f32 {ll}, {lo}, {a_o}
        fma.rn.f32 {ll}, {l}, {a_s}, {ll}
        rcp.rn.f32 {inv}, {ll}
        mul.rn.f32 {cs}, {a_s}, {inv}
        mul.rn.f32 {co}, {a_o}, {inv}
        selp.f32 {c0}, {cs}, {co}, {ph0}
        selp.f32 {c1}, {co}, {cs}, {ph0}
    """)
    bh, q0 = tile_of(c.it)
    oadr, w64 = p.reg("b64"), p.reg("b64")
    grow = p.reg("u32")
    p.emit(f"""
        mad.lo.u32 {grow}, {bh}, {cfg.Sq}, {q0}
        add.u32 {grow}, {grow}, {row}
        mul.wide.u32 {oadr}, {grow}, {cfg.D * 2}
        add.s64 {oadr}, {oadr}, {ptr[cfg.o_param]}
        mul.wide.u32 {w64}, {h}, 128
        add.s64 {oadr}, {oadr}, {w64}
    """)
    oa = [p.reg("b32") for _ in range(32)]
    ob = [p.reg("b32") for _ in range(32)]
    for k in range(2):
        col = p.reg("u32")
        p.emit(f"mad.lo.u32 {col}, {h}, 64, {o_0}")
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(oa)}}}, [{col}+{32 * k}]")
        p.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ob)}}}, [{col}+{128 + 32 * k}]")
        p.emit("tcgen05.wait::ld.sync.aligned")
        fs = []
        for i in range(32):
            fa, fb = p.reg("f32"), p.reg("f32")
            p.emit(f"mov.b32 {fa}, {oa[i]}\nmov.b32 {fb}, {ob[i]}\n"
                   f"mul.rn.f32 {fb}, {fb}, {c1}\nfma.rn.f32 {fa}, {fa}, {c0}, {fb}")
            fs.append(fa)
        pk = [p.reg("b32") for _ in range(16)]
        for i in range(16):
            p.emit(f"{cvt} {pk[i]}, {fs[2 * i + 1]}, {fs[2 * i]}")
        for gg in range(4):
            p.emit(f"st.global.v4.b32 [{oadr}+{(32 * k + 8 * gg) * 2}], {{{', '.join(pk[4 * gg:4 * gg + 4])}}}")
    p.emit("tcgen05.fence::before_thread_sync")
    p.emit(f"mbarrier.arrive.shared::cta.b64 _, [{bar('o_free')}]")
    p.place(l_next)
    c.advance()
    pmore = p.reg("pred")
    p.emit(f"setp.lt.u32 {pmore}, {c.g}, {total}\n@{pmore} bra {l_blk}\nbra {finish}")
