"""The C ABI boundary on the CPU: the shared library loads without a GPU,
exports every function ``include/yabt_b200.h`` declares, the ctypes table in
``yabt_b200/_lib.py`` binds each one with the declared number of arguments, and
the host-only layout functions agree with an independent restatement of the
tiled bin-matrix layout. No compute entry point is called here."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "yabt_b200.h")


def _declarations():
    """(name, n_params) of every function declared in the header."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    out = {}
    for m in re.finditer(r"\b(yabt_[A-Za-z0-9_]+)\s*\(([^;{)]*)\)\s*;", text):
        name, params = m.group(1), m.group(2).strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        out[name] = n
    return out


@pytest.fixture(scope="module")
def lib():
    from yabt_b200 import _lib, build
    if not os.path.exists(_lib.LIB_PATH) or not build.up_to_date():
        build.build()
    return _lib.load()


def test_header_declares_the_path():
    decl = _declarations()
    for name in ("yabt_bin_fit", "yabt_bin_transform", "yabt_grow_tree", "yabt_grow_hist",
                 "yabt_grow_split", "yabt_leafnet_fit", "yabt_update_margin", "yabt_predict_forest",
                 "yabt_hist_build"):
        assert name in decl, name
    assert len(decl) >= 40


def test_library_exports_every_declared_symbol(lib):
    missing = [name for name in _declarations() if not hasattr(lib, name)]
    assert not missing, f"declared in the header but not exported: {missing}"


def test_ctypes_table_matches_header(lib):
    from yabt_b200 import _lib
    decl = _declarations()
    table = {name: args for name, _res, args in _lib.SIGNATURES}
    assert set(table) == set(decl), (set(decl) ^ set(table))
    for name, n in decl.items():
        assert len(table[name]) == n, f"{name}: header has {n} parameters, ctypes table {len(table[name])}"


def test_host_only_queries(lib):
    assert lib.yabt_version() > 0
    assert lib.yabt_bin_fit_static_capacity() == 8 << 20
    # workspace queries are pure arithmetic
    assert lib.yabt_bin_fit_workspace_bytes(200_000, 200, 200_000) > lib.yabt_bin_fit_static_capacity()
    assert lib.yabt_leafnet_workspace_bytes(10_000, 8, 511) > 0
    assert lib.yabt_hist_build_workspace_bytes(20_000, 31, 24) >= 3 * 31 * 24 * 256 * 8 + 20_000 * 4
    assert lib.yabt_hist_build_workspace_bytes(10, 0, 4) < 0
    buf = ctypes.create_string_buffer(64)
    assert lib.yabt_last_error(buf, 64) >= 0


def _expected_layout(n, F):
    """Independent restatement of the tiled layout: 64-feature tiles (lane j of
    a warp reads bytes 2j, 2j+1 = features j and j+32), then one 32-wide tile if
    at least 32 features remain, then a 16- or 32-wide padded tile; every tile
    block starts on a 256-byte boundary."""
    def blk(w):
        return (n * w + 255) // 256 * 256
    addr, off, f = {}, 0, 0
    while F - f >= 64:
        for i in range(64):
            addr[f + i] = (off, 64, 2 * (i % 32) + i // 32)
        off += blk(64)
        f += 64
    if F - f >= 32:
        for i in range(32):
            addr[f + i] = (off, 32, i)
        off += blk(32)
        f += 32
    r = F - f
    if r:
        w = 32 if r > 16 else 16
        for i in range(r):
            addr[f + i] = (off, w, i)
        off += blk(w)
    return addr, off


@pytest.mark.parametrize("n,F", [(1, 1), (1000, 7), (4097, 16), (333, 17), (10_000, 48),
                                 (100, 64), (12345, 100), (10_000_000, 200), (5, 255)])
def test_tiled_layout_addresses(lib, n, F):
    from yabt_b200 import _lib
    addr, total = _expected_layout(n, F)
    assert lib.yabt_bin_matrix_bytes(n, F) == total
    off, width, pos = _lib.c_ll(), ctypes.c_int(), ctypes.c_int()
    for f in range(F):
        assert lib.yabt_bin_address(n, F, f, ctypes.byref(off), ctypes.byref(width), ctypes.byref(pos)) == 0
        assert (off.value, width.value, pos.value) == addr[f], f


def test_struct_layouts_match_header(tmp_path):
    """Every argument struct of the header has the size and field offsets of
    its ctypes mirror in ``yabt_b200/_lib.py`` (a C compiler lays out the
    header's structs; a mismatch would make the library read the wrong bytes)."""
    import shutil
    import subprocess
    from yabt_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    mirrors = {"yabt_tree_args": _lib.TreeArgs, "yabt_leafnet_args": _lib.LeafNetArgs,
               "yabt_update_args": _lib.UpdateArgs}
    lines = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, mirror in mirrors.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in mirror._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src, exe = tmp_path / "layout.c", tmp_path / "layout"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run([cc, "-std=c11", "-o", str(exe), str(src)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, mirror in mirrors.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(mirror), cname
        for field, _ in mirror._fields_:
            assert got[(cname, field)] == getattr(mirror, field).offset, f"{cname}.{field}"


def test_probe_rejects_bad_arguments_before_any_device_call(lib):
    """The measurement probe validates its arguments on the host: unsupported
    limb counts and missing outputs return YABT_ERR_ARG (1) without a GPU."""
    ms, upd = ctypes.c_float(), ctypes.c_longlong()
    for limbs in (0, 4, 6, -1):
        assert lib.yabt_probe_shared_red(limbs, 1, None, None, ctypes.byref(ms), ctypes.byref(upd)) == 1
    for limbs in (1, 2, 3, 5):
        assert lib.yabt_probe_shared_red(limbs, 0, None, None, ctypes.byref(ms), ctypes.byref(upd)) == 1
        assert lib.yabt_probe_shared_red(limbs, 1, None, None, None, None) == 1


def test_level_loop_start_rule(lib):
    """Host-only: the first level of the device-side level loop. The loop runs
    only without level wait, with at least 8 pairs, and when two or more
    levels remain after its first level, which is the first level whose job
    bound 2^(d-1) reaches max_pairs = max_leaves - 1 (at least 4)."""
    def start(leaves, depth, wait=0, loop=1):
        g = ctypes.c_void_p()
        assert lib.yabt_grower_create(1000, 8, leaves, depth, 0, ctypes.byref(g)) == 0
        try:
            assert lib.yabt_grower_set_level_wait(g, wait) == 0
            assert lib.yabt_grower_set_level_loop(g, loop) == 0
            return int(lib.yabt_grower_level_loop_start(g))
        finally:
            lib.yabt_grower_destroy(g)

    def rule(leaves, depth):
        pairs = leaves - 1
        levels = max(1, min(depth, leaves - 1))
        if pairs < 8:
            return -1
        L = 4
        while (1 << (L - 1)) < pairs:
            L += 1
        return L if levels - L >= 2 else -1

    for leaves, depth in ((31, 64), (63, 64), (127, 64), (255, 10), (255, 64), (9, 64), (8, 64), (31, 7), (31, 8),
                          (24, 64), (1000, 12)):
        assert start(leaves, depth) == rule(leaves, depth), (leaves, depth)
    assert start(31, 64) == 6 and start(255, 10) == -1
    assert start(31, 64, wait=1) == -1
    assert start(31, 64, loop=0) == -1
