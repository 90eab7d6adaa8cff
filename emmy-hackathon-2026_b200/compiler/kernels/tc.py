"""sm_100a building blocks shared by the tcgen05 templates (GEMM, attention).

PTX snippets for: mbarrier init / arrive / bounded waits, TMA tile loads, UMMA
shared-memory and instruction descriptors, tcgen05 alloc / mma / commit / ld.

Descriptor formats (PTX ISA, tcgen05 "matrix descriptors"; the same bit layout as
CUTLASS's ``UMMA::SmemDescriptor`` / ``UMMA::InstrDescriptor``):

shared-memory descriptor (64 bit)
  [0,14)  start address >> 4          [16,30) leading-dimension byte offset >> 4
  [32,46) stride-dimension byte offset >> 4
  [46,48) version = 1 (sm_100)         [49,52) base offset (0: 1024-B aligned atoms)
  [52]    LBO mode 0                   [61,64) layout: 0 none, 2 = 128-byte swizzle

  K-major, 128B swizzle: rows of 128 bytes, 8-row atoms 1024 B apart -> SBO = 1024
  (LBO unused, 1).  A K-step of 16 bf16 elements advances the start address by 32 B
  inside the atom; the hardware applies the swizzle to the computed address.
  MN-major, 128B swizzle: 64-element (128 B) MN runs, 8 K-rows per atom -> SBO =
  1024 (next 8 K-rows), LBO = byte distance between 64-element MN blocks.  A
  K-step of 16 advances the start address by 16 rows = 2048 B.

instruction descriptor (32 bit, kind::f16 / kind::f8f6f4)
  [4,6) D format (1 = f32)   [7,10) A format   [10,13) B format
  (kind::f16: 0 = f16, 1 = bf16; kind::f8f6f4: 0 = e4m3, 1 = e5m2)
  [15] A major (0 = K)   [16] B major (1 = MN)   [17,23) N >> 3   [24,29) M >> 4
"""

from __future__ import annotations

TIMEOUT_NS = 2_000_000_000     # every mbarrier wait gives up after 2 s

# status codes written to the kernel's status word when a wait gives up
STATUS = {"producer": 1, "mma": 2, "epilogue": 4, "softmax": 8, "correction": 16, "convert": 32}


def smem_desc_hi(sbo: int, layout: int = 2) -> int:
    """High 32 bits of a shared-memory descriptor: SBO, version 1, layout type."""
    assert sbo % 16 == 0 and (sbo >> 4) < (1 << 14)
    return (sbo >> 4) | (1 << 14) | (layout << 29)


def smem_desc_lo_const(lbo: int) -> int:
    """Low 32 bits without the start address: the LBO field."""
    assert lbo % 16 == 0 and (lbo >> 4) < (1 << 14)
    return (lbo >> 4) << 16


def instr_desc(m: int, n: int, a_fmt: int, b_fmt: int, a_mn_major: bool, b_mn_major: bool,
               d_f32: bool = True) -> int:
    assert m in (64, 128, 256) and n % 8 == 0 and 8 <= n <= 256
    d = (1 if d_f32 else 0) << 4
    d |= a_fmt << 7
    d |= b_fmt << 10
    d |= (1 if a_mn_major else 0) << 15
    d |= (1 if b_mn_major else 0) << 16
    d |= (n >> 3) << 17
    d |= (m >> 4) << 24
    return d


class Waits:
    """Emits bounded mbarrier waits.  On timeout the waiting role records its
    status bit, raises the CTA's abort flag and branches to ``abort_label``;
    any role that sees the abort flag while waiting leaves the same way."""

    def __init__(self, p, status_ptr: str, abort_addr: str):
        self.p = p
        self.status = status_ptr
        self.abort = abort_addr

    def wait(self, bar_addr: str, parity: str, role: str, abort_label: str) -> None:
        p = self.p
        ok, loop, slow, tout = p.label("w_ok"), p.label("w_loop"), p.label("w_slow"), p.label("w_to")
        pw, pa, pt = p.reg("pred"), p.reg("pred"), p.reg("pred")
        t0, t1, ab = p.reg("b64"), p.reg("b64"), p.reg("b32")
        p.emit(f"""
            mbarrier.try_wait.parity.shared::cta.b64 {pw}, [{bar_addr}], {parity}
            @{pw} bra {ok}
            mov.u64 {t0}, %globaltimer
        """)
        p.place(loop)
        p.emit(f"""
            mbarrier.try_wait.parity.shared::cta.b64 {pw}, [{bar_addr}], {parity}
            @{pw} bra {ok}
            ld.volatile.shared.u32 {ab}, [{self.abort}]
            setp.ne.u32 {pa}, {ab}, 0
            @{pa} bra {abort_label}
            mov.u64 {t1}, %globaltimer
            sub.u64 {t1}, {t1}, {t0}
            setp.gt.u64 {pt}, {t1}, {TIMEOUT_NS}
            @!{pt} bra {loop}
        """)
        code = STATUS[role]
        p.emit(f"""
            st.volatile.shared.u32 [{self.abort}], 1
            red.global.or.b32 [{self.status}], {code}
            bra {abort_label}
        """)
        p.place(ok)
