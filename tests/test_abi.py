"""The C ABI: the library loads and exports every function include/helm_b200.h declares; the ctypes
mirrors match the header's structs.  CPU only -- no compute calls."""
import ctypes
import pathlib
import re
import subprocess

import pytest

from helm_b200 import _native as N

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "helm_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(helm_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    fns = declared_functions()
    for name in ("helm_paged_attn_decode", "helm_lse_merge", "helm_int8_linear", "helm_kv_append",
                 "helm_copy_pages", "helm_paged_attn_workspace_bytes", "helm_abi_version", "helm_last_error"):
        assert name in fns


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    assert lib.helm_abi_version() == N.ABI_VERSION
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (helm_[a-z_0-9]+)", out))
    assert set(declared_functions()) <= exported


def test_every_declared_function_has_a_python_signature_or_is_bound_by_its_test():
    bound = {s[0] for s in N.SIGNATURES} | {"helm_paged_attn_decode_noalloc"}
    assert set(declared_functions()) <= bound


def _struct_fields(name):
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    m = re.search(r"typedef struct \{([^{}]*)\}\s*" + name + ";", text)
    body = m.group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        decl = re.sub(r"\s+", " ", decl)
        typ, names = re.match(r"((?:const )?[a-z_0-9]+ ?\*?)\s*(.*)", decl).groups()
        for n in names.split(","):
            n = n.strip().lstrip("*")
            ptr = "*" in typ or n.startswith("*") or "*" in decl.split(n)[0]
            fields.append((n, ptr))
    return fields


@pytest.mark.parametrize("cname,pyname", [("helm_paged_attn_params", "PagedAttnParams"),
                                          ("helm_kv_append_params", "KVAppendParams")])
def test_ctypes_struct_mirrors_header(cname, pyname):
    cfields = [f[0] for f in _struct_fields(cname)]
    pyfields = [f[0] for f in getattr(N, pyname)._fields_]
    assert cfields == pyfields


def test_errors_are_reported_without_a_gpu():
    """Argument validation runs on the host: a bad call returns a status and a message."""
    lib = N.lib()
    p = N.PagedAttnParams()
    p.B, p.Hq, p.Hkv, p.D, p.P = 1, 3, 2, 128, 64   # Hq not a multiple of Hkv
    code = lib.helm_paged_attn_decode(ctypes.byref(p), None)
    assert code == N.ERR_INVALID_ARGUMENT
    assert b"multiple" in lib.helm_last_error()
    code = lib.helm_int8_linear(None, N.F16, None, None, N.F16, None, None, 1, 8, 24, None)
    assert code == N.ERR_UNSUPPORTED
    with pytest.raises(N.HelmError):
        N.check("helm_int8_linear", code)


STRUCTS = [("helm_shard_exchange", "ShardExchange"), ("helm_paged_attn_params", "PagedAttnParams"),
           ("helm_kv_append_params", "KVAppendParams"), ("helm_decode_prologue_params", "DecodePrologueParams"),
           ("helm_gather_merge_params", "GatherMergeParams"), ("helm_kv_prefill_params", "KVPrefillParams")]


def test_ctypes_layouts_match_the_compiled_header(tmp_path):
    """sizeof and every field offset of each ABI struct, as a C compiler lays them out from
    include/helm_b200.h, equal the ctypes mirrors the Python host side passes."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, pyname in STRUCTS:
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in getattr(N, pyname)._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", str(src), "-o", str(exe)], check=True, capture_output=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, pyname in STRUCTS:
        cls = getattr(N, pyname)
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, f"{cname}.{fname}"


def test_move_pages_checks_ids_before_touching_memory():
    """helm_move_pages rejects ids outside the slabs' page counts on the host, before any copy."""
    lib = N.lib()
    src_ids = (ctypes.c_int32 * 2)(0, 5)
    dst_ids = (ctypes.c_int32 * 2)(0, 1)
    n = ctypes.c_int32(-1)
    code = lib.helm_move_pages(ctypes.c_void_p(16), dst_ids, ctypes.c_void_p(16), src_ids, 2, 4096, 4, 5,
                               ctypes.byref(n), None)
    assert code == N.ERR_INVALID_ARGUMENT
    assert b"source page 5" in lib.helm_last_error()
    assert n.value == 0


def test_packed_layout_sizes_and_unpack_on_cpu():
    """helm_int8_packed_bytes and PackedInt8.unpack (torch index arithmetic, no GPU): a weight packed
    by a plain-Python restatement of the documented layout unpacks to itself."""
    import numpy as np
    import torch
    from helm_b200 import ops
    lib = N.lib()
    assert lib.helm_int8_packed_bytes(33, 144) == 3 * 2 * 2048
    assert lib.helm_int8_packed_bytes(16, 24) == -1
    rng = np.random.default_rng(0)
    Nn, K = 37, 272
    w = rng.integers(-127, 128, size=(Nn, K), dtype=np.int8)
    T, KB = -(-Nn // 16), -(-K // 128)
    packed = np.zeros(T * KB * 2048, dtype=np.int8)
    for t in range(T):
        for kb in range(KB):
            for r in range(16):
                for c in range(8):
                    row, k0 = 16 * t + r, 128 * kb + 16 * (c ^ (r & 7))
                    if row < Nn and k0 < K:
                        off = (t * KB + kb) * 2048 + r * 128 + c * 16
                        packed[off:off + 16] = w[row, k0:k0 + 16]
    pk = ops.PackedInt8(torch.from_numpy(packed), Nn, K)
    assert torch.equal(pk.unpack(), torch.from_numpy(w))
    assert torch.equal(ops.int8_pack_weight(torch.from_numpy(w)).data, torch.from_numpy(packed))
    assert torch.equal(pk.rows(16, 37).unpack(), torch.from_numpy(w[16:]))


def _plan(B, Hq, Hkv, pages, splits):
    """(resolved split count, workspace bytes) of helm_paged_attn_workspace_bytes for a bf16 P=64
    D=128 call; host-side planning only (the pointers are never dereferenced)."""
    p = N.PagedAttnParams()
    fake = 1 << 20                                    # 16-byte-aligned stand-in addresses
    p.q, p.k_base, p.v_base, p.out = fake, fake, fake, fake
    p.page_table, p.page_used, p.num_pages = fake, fake, fake
    p.page_stride, p.head_stride = 2 * Hkv * 64 * 128, 64 * 128
    p.num_pool_pages, p.page_table_stride, p.max_pages = B * pages, pages, pages
    p.B, p.Hq, p.Hkv, p.D, p.P = B, Hq, Hkv, 128, 64
    p.q_dtype = p.kv_dtype = p.out_dtype = N.BF16
    p.num_splits = splits
    S = ctypes.c_int32(0)
    need = N.lib().helm_paged_attn_workspace_bytes(ctypes.byref(p), ctypes.byref(S))
    return S.value, need


def test_attention_plan_on_the_host():
    """The automatic plan: k splits per (sequence, kv head) pair, k the largest power of two with
    k * pairs <= 2 * SMs, doubled when every split keeps >= 64 pages; -1 asks for the persistent
    kernel, whose CTA count is a power-of-two multiple of the pairs.  Without a GPU the library
    plans for 148 SMs."""
    rec = lambda S, rows: S * rows * (128 + 2) * 4
    assert _plan(4, 64, 8, 2048, 0) == (16, rec(16, 256))     # config 5: 32 pairs, 2048 pages
    assert _plan(4, 64, 8, 256, 0) == (8, rec(8, 256))        # the N = 8 shard of it
    assert _plan(1, 32, 8, 256, 0) == (32, rec(32, 32))       # batch 1 (config 3's layer)
    assert _plan(4, 64, 8, 2048, 5) == (5, rec(5, 256))       # explicit split count
    S, need = _plan(4, 64, 8, 256, -1)                         # persistent: 8 CTAs per pair = 256
    slots, gq = 256 + 32, 8
    assert S == -1 and need == slots * gq * 128 * 4 + slots * gq * 2 * 4 + 32 * 8
