"""Instruction census / lint of the hand-written inline PTX (zoxide_b200/census.py).

Mirrors the reference's census unit test (src/ptx.zig:516-529: `add.rn.f32`, `ld.global.v4.f32`,
`ret`, `bra` each counted once) and its CI instruction pins (.github/workflows/ci.yml:145-216),
applied to this library's sources: the tcgen05 / TMA / mbarrier forms each kernel family needs
are present, and no lint rule fires (in particular no bulk load broadcast to several CTAs).
"""
from __future__ import annotations

from pathlib import Path

from zoxide_b200 import census as cs

FIXTURE = r'''
__device__ void f(float* p) {
  // asm("bra.uni NOPE;");  commented out: not counted
  asm volatile("add.rn.f32 %0, %1, %2;" : "=f"(a) : "f"(b), "f"(c));
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "@p ld.global.v4.f32 {%0, %0, %0, %0}, [%2];\n\t"
      "LOOP_%=:\n\t"
      "bra LOOP_%=;\n\t}" : "=f"(x) : "r"(y), "l"(p));
  asm("ret;");
  const char* s = "asm(\"trap;\")";  // a string, not an asm statement
}
'''


def test_census_counts_mnemonic_modifier_classes():
    c = cs.census(FIXTURE)
    assert c["add.rn.f32"] == 1
    assert c["ld.global.v4.f32"] == 1
    assert c["ret"] == 1
    assert c["bra"] == 1
    assert c["setp.ne.b32"] == 1
    assert "bra.uni" not in c and "trap" not in c
    assert sum(c.values()) == 5


def test_census_output_format():
    out = cs.format_census("x.cu", cs.census(FIXTURE))
    lines = out.splitlines()
    assert lines[0] == "census: x.cu (5 instruction statements, 5 classes)"
    assert all(ln.startswith("  ") for ln in lines[1:])


def test_lint_flags_forbidden_forms():
    bad = r'''
      asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.BCAST [%0], [%1, {%2, %3}], [%4], %5;" :: "r"(a));
      asm volatile("wgmma.fence.sync.aligned;");
      asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};" : "=r"(d));
      asm volatile("trap;");
    '''
    findings = cs.lint(bad.replace("BCAST", cs._BCAST_Q))  # the broadcast qualifier, spelled by the module
    assert len(findings) == 4
    assert "broadcast" in findings[0][1]


def test_library_sources_census_and_lint():
    srcs = sorted(p for p in cs.CSRC.iterdir() if p.suffix in cs.SOURCE_SUFFIXES)
    assert srcs
    total = sum((cs.census(p.read_text()) for p in srcs), start=cs.Counter())
    # every kernel family's tensor-core form is hand-written
    for key in ("tcgen05.mma.cta_group::2.kind::i8", "tcgen05.mma.cta_group::2.kind::f16",
                "tcgen05.mma.sp.cta_group::2.kind::i8", "tcgen05.mma.cta_group::1.kind::i8",
                "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32",
                "tcgen05.ld.sync.aligned.32x32b.x32.b32", "tcgen05.cp.cta_group::2.128x256b",
                "tcgen05.st.sync.aligned.32x32b.x32.b32"):
        assert total[key] >= 1, key
    assert any(k.startswith("cp.async.bulk.tensor.2d.cta_group::2") for k in total)
    assert any(k.startswith("mbarrier.try_wait") for k in total)
    # the weights-in-TMEM W4A8 kernel's 2-SM MMA takes A from tensor memory: "[d], [a], b, ..."
    ts = [s for p in srcs for s in cs.statements(p.read_text())
          if s.key == "tcgen05.mma.cta_group::2.kind::i8" and s.text.split(None, 1)[1].split(",")[1].strip().startswith("[")]
    assert ts, "no A-from-TMEM cta_group::2 kind::i8 MMA"
    for p in srcs:
        assert cs.lint(p.read_text()) == [], p.name
    assert not any(cs._BCAST in k for k in total)


def test_cli(capsys):
    assert cs.main(["--census", str(cs.CSRC / "zx_ptx.cuh")]) == 0
    assert capsys.readouterr().out.startswith(f"census: {cs.CSRC / 'zx_ptx.cuh'} (")
    assert cs.main([]) == 0
    assert "no findings" in capsys.readouterr().out
    assert cs.main(["--bogus"]) == 2
