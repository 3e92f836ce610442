"""The C ABI library loads without a GPU, exports every entry point include/nsattn.h declares, its
ctypes mirror matches the C struct layouts, and argument validation fails with the documented
status codes before any CUDA call."""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

from nanosaur2_web_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nsattn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nsa_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_library_exports_every_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert _lib.version().startswith("nsattn")
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (nsa_\w+)", out))
    assert set(declared_functions()) <= exported


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layouts_match_c(tmp_path):
    src = tmp_path / "sizes.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "nsattn.h"\n'
                   'int main(){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(nsa_attention_desc),'
                   'offsetof(nsa_attention_desc, b_begin), sizeof(nsa_fused_desc), offsetof(nsa_fused_desc, b_begin),'
                   'sizeof(nsa_kernel_stat), offsetof(nsa_kernel_stat, bytes), sizeof(nsa_seq_shard),'
                   'offsetof(nsa_seq_shard, qkv_text_row0));printf("%zu %zu %zu %zu\\n", sizeof(nsa_proj_desc),'
                   'offsetof(nsa_proj_desc, x_rows), offsetof(nsa_proj_desc, text_rows), offsetof(nsa_proj_desc, b_kv));'
                   'printf("%zu %zu %zu\\n", sizeof(nsa_linear_desc), offsetof(nsa_linear_desc, lda), '
                   'offsetof(nsa_linear_desc, act));printf("%zu %zu %zu\\n", sizeof(nsa_rmsnorm_desc), '
                   'offsetof(nsa_rmsnorm_desc, ldy), offsetof(nsa_rmsnorm_desc, eps));printf("%zu %zu %zu\\n", '
                   'sizeof(nsa_glu_desc), offsetof(nsa_glu_desc, ldy), offsetof(nsa_glu_desc, out_dtype));return 0;}\n')
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(_lib.AttentionDesc), _lib.AttentionDesc.b_begin.offset, ctypes.sizeof(_lib.FusedDesc),
            _lib.FusedDesc.b_begin.offset, ctypes.sizeof(_lib.KernelStat), _lib.KernelStat.bytes.offset,
            ctypes.sizeof(_lib.SeqShard), _lib.SeqShard.qkv_text_row0.offset, ctypes.sizeof(_lib.ProjDesc),
            _lib.ProjDesc.x_rows.offset, _lib.ProjDesc.text_rows.offset, _lib.ProjDesc.b_kv.offset,
            ctypes.sizeof(_lib.LinearDesc), _lib.LinearDesc.lda.offset, _lib.LinearDesc.act.offset,
            ctypes.sizeof(_lib.RmsnormDesc), _lib.RmsnormDesc.ldy.offset, _lib.RmsnormDesc.eps.offset,
            ctypes.sizeof(_lib.GluDesc), _lib.GluDesc.ldy.offset, _lib.GluDesc.out_dtype.offset]
    assert got == want


def _desc(**kw):
    d = _lib.AttentionDesc()
    base = dict(Lq=64, Lk=64, H=2, D=96, ldq=192, ldk=192, ldv=192, group=1, B=1, ldo=192,
                in_dtype=_lib.NSA_BF16, out_dtype=_lib.NSA_F32)
    base.update(kw)
    for k, v in base.items():
        setattr(d, k, v)
    return d


def test_validation_without_gpu():
    L = _lib.lib()
    assert L.nsa_attention(None, None, None, None, None, None, None, None, 0, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    assert b"desc" in L.nsa_last_error()
    fake = 0x10000   # never dereferenced: validation fails first
    cases = [
        (_desc(D=80), _lib.NSA_ERR_UNSUPPORTED),
        (_desc(H=3, group=2), _lib.NSA_ERR_INVALID_ARGUMENT),
        (_desc(in_dtype=7), _lib.NSA_ERR_INVALID_ARGUMENT),
        (_desc(causal=1, Lq=65, Lk=64), _lib.NSA_ERR_INVALID_ARGUMENT),
        (_desc(h_begin=2), _lib.NSA_ERR_INVALID_ARGUMENT),
        (_desc(ldo=190), _lib.NSA_ERR_INVALID_ARGUMENT),
    ]
    for d, want in cases:
        st = L.nsa_attention(ctypes.byref(d), fake, fake, fake, None, None, fake, None, 0, None)
        assert st == want, (st, want, L.nsa_last_error())
    assert L.nsa_head_norm(None, 0, None, 1, 1, 96, 96, 0, 0, None, 0, 1e-6, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    assert L.nsa_rope2d_table(4, 4, 94, fake, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    assert L.nsa_selftest_wait_timeout(0, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    assert L.nsa_status_string(_lib.NSA_ERR_DEVICE) == b"device-side error"


def _split_scratch(units, D, nq=2):
    """Scratch of the tail split: partial O and (m, l) of two half-key CTAs per unit, plus a counter;
    reserved for at most 74 units (half a B200's SMs)."""
    u = min(units, 74)
    up = lambda x: (x + 255) // 256 * 256
    rows = u * 2 * nq * 128
    return up(rows * D * 4) + up(rows * 2 * 4) + up(u * 2 * 4)   # two hand-off counters (query tiles) per unit


def test_workspace_sizes():
    L = _lib.lib()
    d = _desc(Lq=3952, Lk=4208, H=16, D=96, B=2)
    ws = L.nsa_attention_workspace_size(ctypes.byref(d))
    lq_pad, lk_pad = 4096, 4256   # query blocks of 2x128 rows; key tiles of 112 rows for head dim 96
    tiles = 2 * 16 * lq_pad * 96 * 2 + 2 * (2 * 16 * lk_pad * 96 * 2)
    assert ws == tiles + _split_scratch(2 * 16 * 16, 96) + 1024
    d.h_begin, d.h_count = 4, 4
    assert L.nsa_attention_workspace_size(ctypes.byref(d)) == tiles // 4 + _split_scratch(2 * 4 * 16, 96) + 1024
    d.h_begin, d.h_count, d.causal = 0, 0, 1   # causal: no tail split, no scratch
    assert L.nsa_attention_workspace_size(ctypes.byref(d)) == tiles + 1024
    f = _lib.FusedDesc()
    f.B, f.Lq, f.Lk, f.Hq, f.Hkv, f.D, f.causal = 16, 1024, 1024, 4, 1, 256, 1
    wsf = L.nsa_fused_attention_workspace_size(ctypes.byref(f))
    assert wsf == 16 * 4 * 1024 * 256 * 2 + 2 * 16 * 1 * 1024 * 256 * 2 + 1024
    f.D = 100
    assert L.nsa_fused_attention_workspace_size(ctypes.byref(f)) == 0


def test_seq_shard_sizes_and_validation():
    L = _lib.lib()
    d = _lib.FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = 4, 16384, 16640, 16, 16, 96
    d.b_begin, d.b_count = 1, 1
    s = _lib.SeqShard(2048, 2048, 0, 2048)
    qb, kb, rows = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int32()
    st = L.nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(s), ctypes.byref(qb), ctypes.byref(kb),
                                      ctypes.byref(rows))
    assert st == _lib.NSA_OK, L.nsa_last_error()
    assert rows.value == 16688   # 16640 keys rounded up to 112-key tiles
    assert qb.value == 16 * 2048 * 96 * 2 + _split_scratch(16 * 8, 96)
    assert kb.value == rows.value * 2 * 16 * 96 * 2
    fake = 0x10000   # never dereferenced: validation fails first
    d.causal = 1
    assert L.nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(s), None, None, None) == _lib.NSA_ERR_UNSUPPORTED
    assert L.nsa_seq_shard_prologue(ctypes.byref(d), ctypes.byref(s), fake, fake, fake, None, None, fake, fake,
                                    None) == _lib.NSA_ERR_UNSUPPORTED
    d.causal, d.h_begin, d.h_count = 0, 4, 4
    assert L.nsa_seq_shard_attention(ctypes.byref(d), ctypes.byref(s), fake, fake, None, None, fake,
                                     None) == _lib.NSA_ERR_UNSUPPORTED
    d.h_begin, d.h_count = 0, 0
    s.q_begin = 15000   # rows [15000, 17048) run past Lq
    assert L.nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(s), None, None, None) == \
        _lib.NSA_ERR_INVALID_ARGUMENT
    s.q_begin = 0
    assert L.nsa_seq_shard_prologue(ctypes.byref(d), ctypes.byref(s), fake, fake, fake, None, None, fake + 8, fake,
                                    None) == _lib.NSA_ERR_INVALID_ARGUMENT   # q_prime not 16-byte aligned
    assert L.nsa_seq_shard_buffer_sizes(None, ctypes.byref(s), None, None, None) == _lib.NSA_ERR_INVALID_ARGUMENT


def test_projection_and_linear_validation():
    """Argument checks of nsa_seq_shard_projection and nsa_linear (no device work: each case fails
    before any CUDA call)."""
    L = _lib.lib()
    fake = 0x10000   # never dereferenced
    d = _lib.FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = 2, 3952, 4208, 16, 16, 96
    d.in_dtype = d.out_dtype = _lib.NSA_BF16
    s = _lib.SeqShard(0, 3952, 0, 0)
    p = _lib.ProjDesc()
    p.K, p.x, p.ldx, p.x_bstride, p.x_rows, p.w_qkv = 1536, fake, 1536, 3952 * 1536, 3952, fake
    p.x_text, p.ld_text, p.text_bstride, p.text_rows, p.w_kv = fake, 1536, 256 * 1536, 256, fake

    def proj(q_prime=fake):
        return L.nsa_seq_shard_projection(ctypes.byref(d), ctypes.byref(s), ctypes.byref(p), fake, fake, None, None,
                                          q_prime, fake, None)
    assert L.nsa_seq_shard_projection(ctypes.byref(d), ctypes.byref(s), None, fake, fake, None, None, fake, fake,
                                      None) == _lib.NSA_ERR_INVALID_ARGUMENT            # no proj desc
    assert proj(q_prime=fake + 8) == _lib.NSA_ERR_INVALID_ARGUMENT                         # unaligned output
    p.K = 1540
    assert proj() == _lib.NSA_ERR_INVALID_ARGUMENT                                          # K not a multiple of 8
    p.K = 1536
    p.x_text = None
    assert proj() == _lib.NSA_ERR_INVALID_ARGUMENT                                          # text keys need x_text
    p.x_text = fake
    p.text_rows = 100
    assert proj() == _lib.NSA_ERR_INVALID_ARGUMENT                                          # text rows past x_text
    p.text_rows = 256
    d.Hq = d.Hkv = 15
    assert proj() == _lib.NSA_ERR_UNSUPPORTED                                               # heads not whole tiles
    d.Hq = d.Hkv = 16
    d.in_dtype = _lib.NSA_F32
    assert proj() == _lib.NSA_ERR_UNSUPPORTED                                               # bf16 inputs only
    d.in_dtype = _lib.NSA_BF16
    d.causal = 1
    s.q_count = 2000
    assert proj() == _lib.NSA_ERR_UNSUPPORTED                                               # mask over a partial shard
    d.causal, s.q_count = 0, 3952

    ld = _lib.LinearDesc()
    ld.M, ld.N, ld.K, ld.lda = 3952, 1536, 1536, 1536

    def lin(bias=None, gate=None):
        return L.nsa_linear(ctypes.byref(ld), fake, fake, bias, gate, fake, None)
    assert L.nsa_linear(None, fake, fake, None, None, fake, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    ld.N = 1538
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # N not a multiple of 4
    ld.N, ld.lda = 1536, 1000
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # lda < K
    ld.lda = 1536
    assert lin(gate=fake) == _lib.NSA_ERR_INVALID_ARGUMENT                                  # a gate needs resid
    ld.resid, ld.gOff = 1, 2
    assert lin(gate=fake) == _lib.NSA_ERR_INVALID_ARGUMENT                                  # gOff not a multiple of 4
    ld.gOff, ld.act = 0, 3
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # act 0 or 1
    ld.act = 0
    assert lin(bias=fake + 4) == _lib.NSA_ERR_INVALID_ARGUMENT                              # unaligned bias
    ld.resid = 0
    ld.glu = 3
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # glu 0, 1 or 2
    ld.glu, ld.N, ld.ldc = 2, 1664, 832
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # GLU: N not whole tiles
    ld.N, ld.resid = 1536, 1
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # GLU has no resid form
    assert b"fused GLU" in L.nsa_last_error()
    ld.glu, ld.resid, ld.ldc = 0, 0, 0
    ld.schedule = 5
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # unknown schedule
    ld.schedule, ld.M = _lib.NSA_LINEAR_PAIR, 128
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # pairs need M > 128
    assert b"CTA pairs" in L.nsa_last_error()
    ld.M, ld.w_format, ld.w_scale = 3952, _lib.NSA_W_I8, fake
    assert lin() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # pairs: bf16 weights only
    ld.schedule, ld.w_format, ld.w_scale = 0, _lib.NSA_W_BF16, None


def test_rmsnorm_validation():
    """nsa_rmsnorm rejects bad arguments before touching the device (no GPU needed)."""
    L = _lib.lib()
    fake = 1 << 32
    d = _lib.RmsnormDesc()
    d.rows, d.cols, d.eps = 1024, 640, 1e-6

    def rms(x=fake, w=fake + (1 << 28), y=fake + (1 << 30)):
        return L.nsa_rmsnorm(ctypes.byref(d), x, w, y, None)
    assert L.nsa_rmsnorm(None, fake, fake, fake, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    assert rms(w=None) == _lib.NSA_ERR_INVALID_ARGUMENT                                     # missing weight
    d.cols = 0
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # cols >= 1
    d.cols, d.ldx = 640, 600
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # ldx < cols
    d.ldx, d.out_dtype = 0, 7
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # bad dtype
    d.out_dtype, d.accumulate = _lib.NSA_BF16, 1
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # accumulate needs fp32
    d.out_dtype, d.accumulate, d.eps = _lib.NSA_F32, 0, -1.0
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # eps >= 0
    d.eps = 1e-6
    assert rms(y=fake + 4 * 640) == _lib.NSA_ERR_INVALID_ARGUMENT                           # Y overlaps X
    assert b"overlap" in L.nsa_last_error()
    d.next_weight = fake + (1 << 29)
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # next norm needs accumulate
    d.accumulate = 1
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # ... and a Z
    d.Z, d.z_dtype = fake + 64, _lib.NSA_BF16
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # Z overlaps X
    assert b"overlap" in L.nsa_last_error()
    d.Z, d.z_dtype = fake + (1 << 31), 9
    assert rms() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # bad z_dtype
    d.next_weight, d.Z, d.accumulate = None, None, 0
    d.rows = 0
    assert rms(x=None, w=None, y=None) == _lib.NSA_OK                                       # empty: nothing to do


def test_glu_validation():
    """nsa_glu rejects bad arguments before touching the device (no GPU needed)."""
    L = _lib.lib()
    fake = 1 << 32
    d = _lib.GluDesc()
    d.rows, d.I, d.act = 1024, 2048, 1

    def glu(x=fake, y=fake + (1 << 30)):
        return L.nsa_glu(ctypes.byref(d), x, y, None)
    assert L.nsa_glu(None, fake, fake, None) == _lib.NSA_ERR_INVALID_ARGUMENT
    d.ldx = 2048
    assert glu() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # ldx < 2*I
    d.ldx, d.act = 0, 2
    assert glu() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # act 0 or 1
    d.act, d.out_dtype = 1, 5
    assert glu() == _lib.NSA_ERR_INVALID_ARGUMENT                                           # bad dtype
    d.out_dtype = _lib.NSA_F32
    assert glu(y=fake + 4096) == _lib.NSA_ERR_INVALID_ARGUMENT                              # Y overlaps X
    d.rows = 0
    assert glu(x=None, y=None) == _lib.NSA_OK                                               # empty: nothing to do


def test_native_c_caller(tmp_path):
    """A plain C program compiled against include/nsattn.h and linked with libnsattn.so (the way a
    cgo / N-API / JNI host binds it) gets the version string and the same synchronous argument errors
    the Python mirror sees, with messages, and never needs a GPU for them."""
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "nsattn.h"
static int expect(const char* what, nsa_status got, nsa_status want) {
  if (got != want) { printf("FAIL %s: %d (%s)\n", what, (int)got, nsa_last_error()); return 1; }
  printf("ok %s: %s\n", what, nsa_last_error());
  return 0;
}
int main(void) {
  void* p = (void*)0x100000;
  int bad = 0;
  if (strstr(nsa_version(), "sm_100a") == NULL) bad++;
  nsa_attention_desc a; memset(&a, 0, sizeof a);
  a.Lq = a.Lk = 64; a.H = 2; a.D = 80; a.ldq = a.ldk = a.ldv = 160; a.group = 1; a.B = 1; a.ldo = 160;
  bad += expect("attention head dim 80", nsa_attention(&a, p, p, p, NULL, NULL, p, p, 1 << 20, NULL), NSA_ERR_UNSUPPORTED);
  nsa_linear_desc l; memset(&l, 0, sizeof l); l.M = 128; l.N = 256; l.K = 100; l.lda = 100;
  bad += expect("linear K % 8", nsa_linear(&l, p, p, NULL, NULL, (float*)p, NULL), NSA_ERR_INVALID_ARGUMENT);
  nsa_rmsnorm_desc r; memset(&r, 0, sizeof r); r.rows = 8; r.cols = 640; r.out_dtype = NSA_BF16; r.accumulate = 1;
  bad += expect("rmsnorm accumulate into bf16", nsa_rmsnorm(&r, (const float*)p, (const float*)p, (char*)p + (1 << 24), NULL),
                NSA_ERR_INVALID_ARGUMENT);
  nsa_glu_desc g; memset(&g, 0, sizeof g); g.rows = 8; g.I = 16; g.act = 7;
  bad += expect("glu act", nsa_glu(&g, (const float*)p, (char*)p + (1 << 24), NULL), NSA_ERR_INVALID_ARGUMENT);
  bad += expect("rope1d odd D", nsa_rope1d_table(16, 7, 1e4f, (float*)p, NULL), NSA_ERR_INVALID_ARGUMENT);
  bad += expect("status string", strcmp(nsa_status_string(NSA_ERR_DEVICE), "") != 0 ? NSA_OK : NSA_ERR_CUDA, NSA_OK);
  return bad;
}
''')
    exe = tmp_path / "caller"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-L", libdir, "-lnsattn", f"-Wl,-rpath,{libdir}",
                    "-o", str(exe)], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.count("ok ") == 6


def _node_api_include():
    """Directory holding node_api.h (NODE_API_INCLUDE, the usual install prefixes, node-gyp's cache)."""
    cands = [os.environ.get("NODE_API_INCLUDE", ""), "/usr/include/node", "/usr/local/include/node"]
    gyp = os.path.expanduser("~/.cache/node-gyp")
    if os.path.isdir(gyp):
        cands += [os.path.join(gyp, v, "include", "node") for v in sorted(os.listdir(gyp))]
    for c in cands:
        if c and os.path.exists(os.path.join(c, "node_api.h")):
            return c
    return None


@pytest.mark.skipif(shutil.which("gcc") is None or _node_api_include() is None,
                    reason="node_api.h is not installed here (no Node.js toolchain): the addon cannot be compiled")
def test_napi_addon_compiles(tmp_path):
    """The N-API addon (nanosaur2_web_b200/napi/nsattn_addon.c) compiles against node_api.h and the
    library header, as node-gyp would build it."""
    src = os.path.join(ROOT, "nanosaur2_web_b200", "napi", "nsattn_addon.c")
    res = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-fPIC", "-c", "-I", os.path.join(ROOT, "include"),
                          "-I", _node_api_include(), "-DNODE_GYP_MODULE_NAME=nsattn_addon", src, "-o",
                          str(tmp_path / "addon.o")], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_napi_addon_calls_only_declared_entry_points():
    """Every nsa_* function the addon calls is declared in include/nsattn.h (and so exported)."""
    src = open(os.path.join(ROOT, "nanosaur2_web_b200", "napi", "nsattn_addon.c")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    called = set(re.findall(r"\b(nsa_[a-z0-9_]+)\s*\(", src))
    assert called and called <= set(declared_functions())
