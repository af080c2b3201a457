"""The C-ABI library: loads, exports every declared symbol, struct layouts agree,
and the host-only logic (IndexShare, argument checks, workspace sizing)
behaves like the reference. No GPU needed: nothing here launches a kernel."""
import ctypes as C
import os
import re

import pytest

from windlass_b200 import _lib
from windlass_b200._lib import IndexShareC, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "wl_attn.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_ ]*?[\s\*]+(wl_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = header_functions()
    assert len(names) >= 20
    L = lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) == set(_lib.SIGNATURES), "binding and header disagree"


def test_struct_layouts_match_header():
    _lib.check_abi()
    assert lib().wl_abi_version() == 1


def test_strerror_covers_every_status():
    for s in range(10):
        assert lib().wl_strerror(s).decode() not in ("", "unknown status")
    assert lib().wl_strerror(99).decode() == "unknown status"


def _cfg(T=4096):
    cfg = _lib.AttnCfg()
    lib().wl_attn_cfg_glm52(C.byref(cfg), T)
    return cfg


def test_glm52_config_values():
    c = _cfg()
    assert (c.n_heads, c.kv_lora, c.rope_dim, c.idx_heads, c.idx_dim, c.index_topk) == (64, 512, 64, 32, 128, 2048)
    assert c.softmax_scale == pytest.approx(256 ** -0.5)
    assert c.idx_qk_scale == pytest.approx(128 ** -0.5)


# ---- IndexShare (glm_layer_runner.cuh:485-517; test_glm_index_share.cu:60-237) ----

def glm_ownership(n_layers):
    """Owners at 0, 1, 2, 6, 10, ...: (max(i-2, 0) % 4) == 0 (test_glm_index_share.cu:79-92)."""
    owner, leader, cur = [], [], None
    for i in range(n_layers):
        m = i - 2 if i >= 2 else 0
        owner.append(m % 4 == 0)
        if owner[-1]:
            cur = i
        leader.append(cur)
    return owner, leader


def walk_group(n_layers, clear_after_use=False):
    """Run the layer loop's share protocol with unique fake pointers per owner;
    returns the list of (layer, pointer seen) or raises on a violation."""
    owner, leader = glm_ownership(n_layers)
    s = IndexShareC()
    lib().wl_index_share_reset(C.byref(s))
    seen = []
    for layer in range(n_layers):
        if owner[layer]:
            lib().wl_index_share_publish(C.byref(s), layer, 0x1000 * (layer + 1), None, 2048, 2048)
            seen.append((layer, s.idx))
        else:
            st = lib().wl_index_share_require(C.byref(s), layer)
            if st != _lib.WL_OK:
                raise RuntimeError(f"layer {layer}: {st}")
            seen.append((layer, s.idx))
            assert s.producer == leader[layer]
            if clear_after_use:
                lib().wl_index_share_reset(C.byref(s))
    return seen, leader


def test_index_share_propagates_across_whole_group():
    seen, leader = walk_group(78)
    for layer, ptr in seen:
        assert ptr == 0x1000 * (leader[layer] + 1)


def test_index_share_negative_control_consume_and_clear():
    with pytest.raises(RuntimeError):
        walk_group(78, clear_after_use=True)


def test_shared_layer_with_nothing_published_fails():
    s = IndexShareC()
    lib().wl_index_share_reset(C.byref(s))
    assert lib().wl_index_share_require(C.byref(s), 3) == _lib.WL_ERR_NO_INDICES
    s.dense = 1
    assert lib().wl_index_share_require(C.byref(s), 3) == _lib.WL_OK


def test_python_index_share_raises_like_reference():
    from windlass_b200.attn import IndexShare
    s = IndexShare()
    with pytest.raises(RuntimeError, match="no published indices"):
        s.require(5)
    assert IndexShare(dense=True).require(5) is None


def test_reset_keeps_dense_mode_and_clears_indices():
    s = IndexShareC()
    s.dense = 1
    lib().wl_index_share_publish(C.byref(s), 2, 0x10, None, 8, 8)
    lib().wl_index_share_reset(C.byref(s))
    assert s.idx is None and s.producer == 0xFFFFFFFF and s.dense == 1


# ---- argument checking and sizing (return before any CUDA call) ----

def test_decode_rejects_bad_arguments_without_touching_the_gpu():
    cfg = _cfg(1024)
    io = _lib.DecodeIO()
    assert lib().wl_attn_decode(C.byref(cfg), None, None, 0, None) == _lib.WL_ERR_ARG
    io.batch, io.T = 1, 2048
    io.q_abs, io.ctx = 16, 16
    io.mode = _lib.WL_MODE_DENSE
    assert lib().wl_attn_decode(C.byref(cfg), C.byref(io), None, 0, None) == _lib.WL_ERR_T_EXCEEDS_MAX
    io.T = 512
    io.mode = _lib.WL_MODE_CONSUMER
    assert lib().wl_attn_decode(C.byref(cfg), C.byref(io), None, 0, None) == _lib.WL_ERR_NO_INDICES
    io.mode = _lib.WL_MODE_DENSE
    assert lib().wl_attn_decode(C.byref(cfg), C.byref(io), None, 0, None) == _lib.WL_ERR_WORKSPACE
    bad = _cfg(1024)
    bad.n_heads = 128
    assert lib().wl_attn_decode(C.byref(bad), C.byref(io), None, 0, None) == _lib.WL_ERR_UNSUPPORTED


def test_workspace_sizes_scale_with_batch_and_T():
    cfg = _cfg(131072)
    a = lib().wl_attn_workspace_bytes(C.byref(cfg), 32768, 1)
    b = lib().wl_attn_workspace_bytes(C.byref(cfg), 32768, 8)
    c = lib().wl_attn_workspace_bytes(C.byref(cfg), 131072, 1)
    assert 0 < a < b and a < c
    # scores + selection + 16 split partials of 64x512 fp32 per sequence
    assert a >= 32768 * 4 + 16 * 64 * 512 * 4
    s = lib().wl_attn_sharded_workspace_bytes(C.byref(cfg), 4096, 8, 8)
    assert s > lib().wl_attn_workspace_bytes(C.byref(cfg), 4096, 8)
    assert lib().wl_attn_prefill_workspace_bytes(C.byref(cfg), 4096, 8192) >= 4096 * 8192 * 4


# ---- argument checks of the entry points around the substep (no launch happens) ----

def test_cache_append_argument_checks():
    cfg = _cfg()
    io = _lib.CacheAppendIO()
    io.n = 0
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_OK  # nothing to do
    io.n = 4
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG  # no pos / tables
    io.pos, io.cos, io.sin = 0x1000, 0x2000, 0x3000
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG  # neither part given
    io.k_raw = 0x4000
    io.n_seq = 0  # the caches must hold at least one sequence
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG
    io.seq, io.n_seq = None, 2  # without a sequence list there is exactly one
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG
    io.n_seq = 1
    io.k_raw = 0x4008  # misaligned, and no cache / norm weights
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG
    io.n = -1
    assert lib().wl_cache_append(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_ARG
    bad = _cfg()
    bad.kv_lora = 256
    assert lib().wl_cache_append(C.byref(bad), C.byref(io), None) == _lib.WL_ERR_UNSUPPORTED


def test_projection_argument_checks():
    cfg = _cfg()
    L = lib()
    assert L.wl_mla_absorb_q(C.byref(cfg), 0, None, 0, None, None, 0, None) == _lib.WL_OK
    assert L.wl_mla_absorb_q(C.byref(cfg), 2, None, 64 * 256, 0x1000, 0x2000, 64 * 576, None) == _lib.WL_ERR_ARG
    assert L.wl_mla_absorb_q(C.byref(cfg), 2, 0x1000, 100, 0x1000, 0x2000, 64 * 576, None) == _lib.WL_ERR_ARG
    assert L.wl_mla_project_v(C.byref(cfg), 0, None, 0, None, None, 0, None) == _lib.WL_OK
    assert L.wl_mla_project_v(C.byref(cfg), 1, 0x1000, 64 * 512, 0x2008, 0x3000, 64 * 256, None) == _lib.WL_ERR_ARG
    assert L.wl_mla_project_v(C.byref(cfg), -1, 0x1000, 64 * 512, 0x2000, 0x3000, 64 * 256, None) == _lib.WL_ERR_ARG
    q = dict(q_resid=0x1000, wq_b=0x2000, x=0x3000, wp=0x4000, cos=0x5000, sin=0x6000, qi=0x7000, wi=0x8000)
    args = lambda hidden, n=1: (C.byref(cfg), n, q["q_resid"], 2048, q["wq_b"], q["x"], hidden, hidden,  # noqa: E731
                                q["wp"], q["cos"], q["sin"], q["qi"], q["wi"], None)
    assert L.wl_indexer_query(*args(1000)) == _lib.WL_ERR_ARG  # hidden not a multiple of 1024
    assert L.wl_indexer_query(*args(6144, n=0)) == _lib.WL_OK
    assert L.wl_indexer_query(C.byref(cfg), 1, None, 2048, 0x2000, 0x3000, 6144, 6144, 0x4000, 0x5000, 0x6000,
                              0x7000, 0x8000, None) == _lib.WL_ERR_ARG


def test_layer_prefill_requires_a_published_share():
    from windlass_b200._lib import PrefillIO
    cfg = _cfg()
    s = IndexShareC()
    lib().wl_index_share_reset(C.byref(s))
    io = PrefillIO()
    io.n_q, io.pos0 = 4, 100
    assert lib().wl_attn_layer_prefill(C.byref(cfg), C.byref(io), 0, 3, C.byref(s), None, 0, None) \
        == _lib.WL_ERR_NO_INDICES
    # an owner must name the buffers it publishes
    assert lib().wl_attn_layer_prefill(C.byref(cfg), C.byref(io), 1, 3, C.byref(s), None, 0, None) \
        == _lib.WL_ERR_ARG


def test_header_compiles_as_c_and_links(tmp_path):
    """The boundary is a C ABI: include/wl_attn.h compiles as C99, and a C
    program links against libwl_attn.so and runs its host-only calls."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "probe.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "wl_attn.h"
int main(void) {
    wl_attn_cfg cfg;
    wl_attn_cfg_glm52(&cfg, 4096);
    if (cfg.n_heads != 64 || cfg.kv_lora != 512 || cfg.index_topk != 2048) return 1;
    if (strcmp(wl_strerror(WL_OK), "unknown status") == 0) return 2;
    wl_index_share s;
    memset(&s, 0, sizeof s);
    wl_index_share_reset(&s);
    if (wl_index_share_require(&s, 3) != WL_ERR_NO_INDICES) return 3;
    wl_index_share_publish(&s, 0, (const int32_t*)0x100, NULL, 8, 8);
    if (wl_index_share_require(&s, 3) != WL_OK || s.producer != 0) return 4;
    wl_cache_append_io a;
    memset(&a, 0, sizeof a);
    a.n = 1;
    if (wl_cache_append(&cfg, &a, NULL) != WL_ERR_ARG) return 5;
    if (wl_abi_version() != WL_ABI_VERSION) return 6;
    printf("ok\n");
    return 0;
}
""")
    exe = tmp_path / "probe"
    libdir = os.path.join(ROOT, "windlass_b200")
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-L", libdir,
                    "-l:libwl_attn.so", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", (out.returncode, out.stdout, out.stderr)


def test_noalloc_rejections_happen_before_any_device_work():
    """wl_attn_decode_noalloc refuses, with WL_ERR_UNSUPPORTED, the two modes
    that would need scratch beyond its fixed array (an owner layer's indexer
    and top-k; normalising a non-canonical list), and batches past its
    maximum with WL_ERR_WORKSPACE — all before touching the GPU."""
    cfg = _cfg()
    io = _lib.DecodeIO()
    io.batch, io.T = 1, 100
    io.q_abs, io.ctx = 0x1000, 0x2000
    io.mode = _lib.WL_MODE_OWNER
    io.q_idx, io.w_idx = 0x3000, 0x4000
    io.index.keys, io.index.scale = 0x5000, 0x6000
    L = lib()
    assert L.wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_UNSUPPORTED
    io.mode = _lib.WL_MODE_CONSUMER
    io.sel_in, io.sel_n, io.sel_stride, io.sel_flags = 0x7000, 10, 10, 0
    assert L.wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_UNSUPPORTED
    io.sel_flags = _lib.WL_SEL_CANONICAL
    io.batch = 5
    assert L.wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_WORKSPACE
    io.sel_in = None  # a consumer with nothing to consume
    assert L.wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), None) == _lib.WL_ERR_NO_INDICES
