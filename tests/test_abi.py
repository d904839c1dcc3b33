"""The C-ABI library builds, loads and exports every entry point that
include/nkv.h declares. CPU only: no compute calls."""

import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _header_functions() -> list[str]:
    text = (REPO / "include" / "nkv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nkv_[a-z_0-9]+)\s*\(", text)))


def test_library_builds_and_exports_every_symbol():
    from nanokv_b200 import _lib, build

    build.build()
    lib = _lib.load()
    declared = _header_functions()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in nkv.h but not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes bindings out of sync with nkv.h"
    assert lib.nkv_abi_version() == 102
    assert lib.nkv_status_string(3) == b"NKV_ERR_WORKSPACE"


def test_workspace_query_is_pure_host():
    from nanokv_b200 import _lib

    lib = _lib.load()
    n = lib.nkv_paged_decode_workspace_size(256, 32, 8, 128, 32, 256)
    assert n > 0 and n % 256 == 0
    assert lib.nkv_paged_decode_workspace_size(256, 30, 8, 128, 32, 256) == 0  # Hq % Hk != 0


def test_argument_errors_need_no_gpu():
    """Validation happens before any CUDA call, so it is testable on CPU."""
    from nanokv_b200 import _lib

    lib = _lib.load()
    # unsupported head_dim
    assert lib.nkv_paged_decode(16, 0, 0, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 64, 256,
                                0.1, 16, 1 << 20, None) == 2
    # workspace too small
    assert lib.nkv_paged_decode(16, 4096, 128, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 128, 256,
                                0.1, 16, 8, None) == 3
    # misaligned q
    assert lib.nkv_paged_decode(18, 4096, 128, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 128, 256,
                                0.1, 16, 1 << 30, None) == 4
    # zero tokens is a no-op for the store
    assert lib.nkv_store_kvcache(16, 1024, 16, 1024, 16, 16, 100, 16, 0, 8, 128, None) == 0
    # obs_window other than 1 is not the reference's periodic path
    assert lib.nkv_window_compress(16, 4096, 16, 16, 10, 16, 8, 16, 16, 16, 1, 4, 513, 2, 32, 8,
                                   128, 256, 0.1, None, None, None, None) == 2


def test_prefill_argument_errors_need_no_gpu():
    """nkv_paged_prefill validates shapes, strides and alignment on the host."""
    from nanokv_b200 import _lib

    lib = _lib.load()
    base = dict(q=16, qst=4096, qsh=128, nq=100, k=16, kst=1024, v=16, vst=1024, rows=1000,
                bt=16, mb=8, bs=256, cuq=16, cuk=16, b=2, mq=64, causal=1, out=16, ost=4096,
                hq=32, hk=8, d=128, scale=0.1, stream=None)

    def call(**over):
        a = dict(base, **over)
        return lib.nkv_paged_prefill(*a.values())

    assert call(d=64) == 2                      # head_dim 128 only
    assert call(bs=100) == 2                    # paged block size multiple of 64
    assert call(q=18) == 4                      # misaligned q
    assert call(kst=1028) == 4                  # row stride not a 16-byte multiple
    assert call(hq=30) == 1                     # Hq % Hk != 0
    assert call(ost=2048) == 1                  # out rows too short for Hq heads
    assert call(b=0) == 0 and call(mq=0) == 0   # empty batch is a no-op
    assert call(scale=float("inf")) == 1
    assert call(scale=-0.1) == 1


def test_norm_rope_argument_errors_need_no_gpu():
    from nanokv_b200 import _lib

    lib = _lib.load()
    base = dict(qkv=16, qst=6144, T=4, pos=16, cs=16, maxp=128, qw=16, kw=16, eps=1e-6, qo=16,
                qost=4096, ko=None, kost=0, kc=None, vc=None, ns=0, sm=None, hq=32, hk=8, d=128,
                stream=None)

    def call(**over):
        a = dict(base, **over)
        return lib.nkv_qk_norm_rope_store(*a.values())

    assert call(d=64) == 2                  # head_dim 128 only
    assert call(qkv=24) == 4                # rows not 16-byte aligned
    assert call(qst=6000) == 1              # row shorter than (Hq + 2 Hk) * D
    assert call(cs=24) == 4                 # cos/sin cache must be 16-byte aligned
    assert call(kc=16) == 1                 # cache without v_cache / slot_mapping
    assert call(T=0) == 0


def _header_prototypes() -> dict[str, list[str]]:
    """name -> parameter type strings, parsed from include/nkv.h."""
    text = (REPO / "include" / "nkv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    protos = {}
    for m in re.finditer(r"\b(nkv_[a-z_0-9]+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(2).split(",") if p.strip()]
        if params == ["void"]:
            params = []
        # drop the parameter name: the type is everything before the last word
        protos[m.group(1)] = [re.sub(r"\s*\b\w+$", "", p).strip() for p in params]
    return protos


def _ctypes_kind(ct) -> str:
    import ctypes
    if ct in (ctypes.c_void_p, ctypes.c_char_p) or hasattr(ct, "contents") or \
            getattr(ct, "_type_", None) is not None and ct.__name__.startswith("LP_"):
        return "ptr"
    size = ctypes.sizeof(ct)
    if ct in (ctypes.c_float,):
        return "f32"
    if ct in (ctypes.c_double,):
        return "f64"
    return f"int{size * 8}"


def _c_kind(t: str) -> str:
    if "*" in t:
        return "ptr"
    t = t.replace("const", "").strip()
    return {"float": "f32", "double": "f64", "int": "int32", "int32_t": "int32",
            "uint32_t": "int32", "int64_t": "int64", "uint64_t": "int64", "size_t": "int64",
            "unsigned": "int32", "unsigned int": "int32"}.get(t, "?" + t)


def test_ctypes_argtypes_match_header_prototypes():
    """Every binding in _lib.SIGNATURES has the prototype's parameter count,
    and each parameter's kind (pointer / 32- or 64-bit integer / float)
    matches the header's type, so the ABI cannot drift silently."""
    from nanokv_b200 import _lib

    protos = _header_prototypes()
    assert set(protos) == set(_lib.SIGNATURES)
    for name, (_, argtypes) in _lib.SIGNATURES.items():
        ctypes_kinds = [_ctypes_kind(a) for a in argtypes]
        c_kinds = [_c_kind(t) for t in protos[name]]
        assert len(ctypes_kinds) == len(c_kinds), (name, len(ctypes_kinds), len(c_kinds))
        assert ctypes_kinds == c_kinds, (name, list(zip(c_kinds, ctypes_kinds)))


def test_newer_entry_points_validate_before_any_cuda_call():
    """Status codes (no exceptions across the ABI) for the prefill, q/k
    norm + RoPE, device selection and o_proj entries, from argument checks
    that run before any CUDA call. Status: 0 ok, 1 invalid argument,
    2 unsupported, 4 alignment."""
    from nanokv_b200 import _lib

    lib = _lib.load()
    OK, INVALID, UNSUPPORTED, ALIGN = 0, 1, 2, 4
    nan = float("nan")

    def prefill(**kw):
        a = dict(q=4096, qst=4096, qsh=128, T=16, k=4096, kst=1024, v=8192, vst=1024, rows=256,
                 bt=None, mb=0, bs=0, cuq=16, cuk=16, batch=1, maxq=16, causal=1, out=4096,
                 ost=4096, hq=32, hk=8, d=128, scale=0.088)
        a.update(kw)
        return lib.nkv_paged_prefill(a["q"], a["qst"], a["qsh"], a["T"], a["k"], a["kst"], a["v"],
                                     a["vst"], a["rows"], a["bt"], a["mb"], a["bs"], a["cuq"],
                                     a["cuk"], a["batch"], a["maxq"], a["causal"], a["out"],
                                     a["ost"], a["hq"], a["hk"], a["d"], a["scale"], None)

    assert prefill(batch=0) == OK
    assert prefill(hq=30) == INVALID          # Hq not a multiple of Hk
    assert prefill(scale=nan) == INVALID
    assert prefill(d=64) == UNSUPPORTED
    assert prefill(bt=16, mb=4, bs=100) == UNSUPPORTED  # 128-key tiles need 64 or k*128
    assert prefill(q=4098) == ALIGN
    assert prefill(ost=100) == INVALID         # output rows shorter than Hq * 128

    def norm_rope(**kw):
        a = dict(qkv=4096, st=6144, T=4, pos=16, cs=4096, maxpos=1024, qw=4096, kw=4096, eps=1e-6,
                 qo=4096, qost=4096, ko=None, kost=0, kc=None, vc=None, ns=0, sm=None, hq=32,
                 hk=8, d=128)
        a.update(kw)
        return lib.nkv_qk_norm_rope_store(a["qkv"], a["st"], a["T"], a["pos"], a["cs"],
                                          a["maxpos"], a["qw"], a["kw"], a["eps"], a["qo"],
                                          a["qost"], a["ko"], a["kost"], a["kc"], a["vc"],
                                          a["ns"], a["sm"], a["hq"], a["hk"], a["d"], None)

    assert norm_rope(T=0) == OK
    assert norm_rope(d=64) == UNSUPPORTED
    assert norm_rope(eps=-1.0) == INVALID
    assert norm_rope(kc=4096, vc=8192, ns=64) == INVALID   # a cache needs its slot_mapping
    assert norm_rope(st=100) == INVALID
    assert norm_rope(qkv=4098) == ALIGN

    assert lib.nkv_window_select(16, 16, -1, 256, 4, 2, 16, None, None, None) == INVALID
    assert lib.nkv_window_select(None, None, 0, 256, 4, 0, None, None, None, None) == OK
    assert lib.nkv_window_select(16, 16, 2, 256, 4, 2, None, None, None, None) == INVALID

    def oproj(**kw):
        a = dict(x=4096, ldx=512, w=8192, ldw=512, T=16, k=512, n=1024, pmc=4096, pl=4096,
                 omc=4096, ol=4096, smc=4096, sl=4096, flags=4096, rank=0, world=2, to=10**9,
                 ws=4096, wsb=1 << 20, y=4096, ldy=1024)
        a.update(kw)
        return lib.nkv_oproj_allreduce(a["x"], a["ldx"], a["w"], a["ldw"], a["T"], a["k"], a["n"],
                                       a["pmc"], a["pl"], a["omc"], a["ol"], a["smc"], a["sl"],
                                       a["flags"], a["rank"], a["world"], a["to"], a["ws"],
                                       a["wsb"], a["y"], a["ldy"], None)

    assert oproj(T=0) == OK
    assert oproj(rank=2) == INVALID
    assert oproj(pl=None) == INVALID
    assert oproj(k=100) == UNSUPPORTED
    assert oproj(T=513) == UNSUPPORTED         # decode-sized steps only
    assert oproj(ldy=100) == INVALID
    assert oproj(x=4098) == ALIGN

    def p2p(**kw):
        a = dict(x=4096, ldx=512, w=8192, ldw=512, T=16, k=512, n=1024, rp=4096, ss=16 * 1024,
                 sp=4096, sl=4096, flags=4096, rank=0, world=2, to=10**9, ws=4096, wsb=1 << 20,
                 y=4096, ldy=1024)
        a.update(kw)
        return lib.nkv_oproj_allreduce_p2p(a["x"], a["ldx"], a["w"], a["ldw"], a["T"], a["k"],
                                           a["n"], a["rp"], a["ss"], a["sp"], a["sl"], a["flags"],
                                           a["rank"], a["world"], a["to"], a["ws"], a["wsb"],
                                           a["y"], a["ldy"], None)

    assert p2p(T=0) == OK
    assert p2p(rp=None) == INVALID
    assert p2p(ss=16 * 1024 - 8) == INVALID    # a slot must hold tokens x n
    assert p2p(ss=16 * 1024 + 4) == ALIGN      # slots start on 16 bytes
    assert p2p(world=0) == INVALID
