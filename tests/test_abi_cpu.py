"""The C ABI library loads without a GPU, exports every declared entry point,
and rejects bad scalar arguments on the host before launching anything."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from vllm_ascend_kvcompress import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "kvc.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(kvc_\w+)\(", text, re.M))


def test_library_loads_and_reports_abi_version():
    lib = N.lib()
    assert lib.kvc_abi_version() == N.ABI_VERSION


def test_every_declared_symbol_is_exported_and_bound():
    lib = N.lib()
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), s
    assert syms == set(N.exported_symbols())


def test_status_strings():
    lib = N.lib()
    assert lib.kvc_status_string(0) == b"ok"
    assert b"NULL" in lib.kvc_status_string(-14)


def test_coef_floats_layout():
    lib = N.lib()
    assert lib.kvc_coef_floats(64, 5, 17, 0) == 64 * 16
    assert lib.kvc_coef_floats(32, 8, 17, 0) == 32 * 24
    assert lib.kvc_coef_floats(64, 5, 17, 1) == 64 * 16 + 17 * 64 * 10


def test_fragment_record_and_scorer_geometries():
    """Per (request, layer, KV head): 16-bit coefficients of 4F + P rows x 16
    columns, then one 16-byte record holding the inverse W scale."""
    lib = N.lib()
    assert lib.kvc_fragment_words(64, 0) == (4 * 64 * 16 * 2 + 16) // 4
    assert lib.kvc_fragment_words(32, 192) == ((4 * 32 + 192) * 16 * 2 + 16) // 4
    assert lib.kvc_fragment_words(30, 0) == 0  # F must be a multiple of 16
    # the mma.sync scorer instantiates head_dim 256 full RoPE; the tcgen05 one
    # (512 TMEM columns over three warpgroups) does not
    assert lib.kvc_tc_supported(5, 128, 128) == 1 and lib.kvc_tc05_supported(5, 128, 128) == 1
    assert lib.kvc_tc_supported(8, 256, 64) == 1 and lib.kvc_tc05_supported(8, 256, 64) == 1
    assert lib.kvc_tc_supported(4, 256, 256) == 1 and lib.kvc_tc05_supported(4, 256, 256) == 0
    assert lib.kvc_tc05_supported(9, 128, 128) == 0  # query group above 8
    assert lib.kvc_tc05_supported(5, 128, 127) == 0  # odd rotary dim
    assert lib.kvc_tc_partials_per_page() == 4


def test_host_validation_rejects_without_launch():
    lib = N.lib()
    fake = ctypes.c_void_p(0x1000)
    # NULL pointers
    assert lib.kvc_select_keep(None, None, None, 1, 10, 0, 0, 8, 1, None, None, None) == -14
    # budget 0 / windows larger than the budget / unknown policy
    assert lib.kvc_select_keep(fake, fake, fake, 1, 0, 0, 0, 8, 1, fake, None, None) == -22
    assert lib.kvc_select_keep(fake, fake, fake, 1, 10, 6, 6, 8, 1, fake, None, None) == -22
    assert lib.kvc_select_keep(fake, fake, fake, 1, 10, 0, 0, 8, 7, fake, None, None) == -22
    # score: query group above the compiled maximum
    ptrs = N.pointer_array([0x100000])
    rc = lib.kvc_score_paged_keys(ptrs, 1, 0, 128 * 8 * 128, 10, 8, 9, 128, 128, fake, fake, fake, fake, 1, 1,
                                  fake, 17, 0, None, fake, fake, None, None)
    assert rc in (-22, -95)
    # score: frequency count not a multiple of 8 on the streaming (mean) kernel
    rc = lib.kvc_score_paged_keys(ptrs, 1, 0, 128 * 8 * 4, 10, 8, 4, 4, 4, fake, fake, fake, fake, 1, 1,
                                  fake, 17, 0, None, fake, fake, None, None)
    assert rc == -95
    # compaction: misaligned layer pointer (odd address)
    k = N.pointer_array([0x100001])
    v = N.pointer_array([0x200000])
    rc = lib.kvc_compact(k, v, 1, 128 * 2048, 10, 2048, fake, fake, fake, fake, fake, fake, 1, 128,
                         None, 0, None, None, None, None)
    assert rc == -71
    # compaction: block stride smaller than a page
    rc = lib.kvc_compact(N.pointer_array([0x100000]), v, 1, 1024, 10, 2048, fake, fake, fake, fake, fake, fake,
                         1, 128, None, 0, None, None, None, None)
    assert rc == -22
    # calibration: rotary dim above head dim; workspace too small
    assert lib.kvc_calibration_accumulate(fake, 0, 10, 64, 1, 64, 128, fake, fake, fake, None, fake, 1000,
                                          None) == -22
    assert lib.kvc_calibration_accumulate(fake, 0, 10000, 64, 1, 64, 64, fake, fake, fake, None, fake, 1,
                                          None) == -22
    # shift positions: bad index width
    assert lib.kvc_shift_positions(fake, fake, 2, fake, 1, 1, fake, None, None) == -22


def test_check_raises_with_status_text():
    with pytest.raises(RuntimeError, match="EINVAL"):
        N.check(-22, "kvc_test")


def test_kernels_refuse_cpu_tensors():
    import torch

    from vllm_ascend_kvcompress.methods.triattention import kernels as K
    from vllm_ascend_kvcompress.methods.triattention.selection import select_keep_indices

    with pytest.raises(RuntimeError, match="CUDA"):
        select_keep_indices(torch.arange(16.0), budget=12, protected_prefix=2, protected_recent=2, segments=4,
                            policy="v3")
    with pytest.raises(RuntimeError, match="CUDA"):
        K.require_cuda(torch.zeros(1))


def test_step_descriptor_matches_header_field_for_field():
    body = re.search(r"typedef struct kvc_triattention_step \{(.*?)\} kvc_triattention_step;", HEADER.read_text(),
                     re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = re.findall(r"(\w+)\s*;", body)
    assert fields == [f for f, _ in N.TriAttentionStep._fields_]
    assert N.lib().kvc_triattention_step_size() == ctypes.sizeof(N.TriAttentionStep)
    for name, ctype in N.TriAttentionStep._fields_:
        decl = re.search(r"([\w\s\*]+?)\b" + name + r"\s*;", body).group(1)
        assert ("*" in decl) == (ctype is ctypes.c_void_p), name
        if ctype is not ctypes.c_void_p:
            assert decl.split()[-1] == {ctypes.c_int32: "int32_t", ctypes.c_int64: "int64_t"}[ctype], name


def test_step_rejects_bad_stage_masks_without_launch():
    lib = N.lib()
    st = N.TriAttentionStep()
    assert lib.kvc_triattention_run(None, N.STAGE_ALL, None, None) == -14
    assert lib.kvc_triattention_run(ctypes.byref(st), 0, None, None) == -22
    assert lib.kvc_triattention_run(ctypes.byref(st), 64, None, None) == -22
    assert lib.kvc_triattention_run(ctypes.byref(st), N.STAGE_EXCHANGE | N.STAGE_AGGREGATE, None, None) == -22
    assert lib.kvc_triattention_run(ctypes.byref(st), N.STAGE_EXCHANGE, None, None) == -14  # no peer tables
    assert lib.kvc_triattention_run(ctypes.byref(st), N.STAGE_TABLES, None, None) == -14


def test_exchange_ipc_and_unrotate_validate_on_the_host():
    lib = N.lib()
    fake = ctypes.c_void_p(0x1000)
    assert lib.kvc_tp_exchange_flag_words(8) == 28 and lib.kvc_tp_exchange_flag_words(0) == 0
    assert lib.kvc_tp_exchange_stamp_word(8) == 20 and lib.kvc_tp_exchange_stamp_word(8) % 2 == 0
    # inbox: 8 sources x 6 layers x ceil(1000 pages * 32 quads / 8) quads x 4 floats
    assert lib.kvc_tp_exchange_inbox_floats(8, 6, 1000) == 8 * 6 * 4000 * 4
    # exchange: NULL tables, rank outside the world, world above the maximum, epoch 0, bad aggregation
    assert lib.kvc_tp_exchange_max(None, fake, fake, 2, 0, 1, 1, fake, fake, 1, 0, 1, None, None) == -14
    assert lib.kvc_tp_exchange_max(fake, fake, fake, 2, 2, 1, 1, fake, fake, 1, 0, 1, None, None) == -22
    assert lib.kvc_tp_exchange_max(fake, fake, fake, N.TP_MAX_WORLD + 1, 0, 1, 1, fake, fake, 1, 0, 1, None,
                                   None) == -22
    assert lib.kvc_tp_exchange_max(fake, fake, fake, 2, 0, 1, 1, fake, fake, 1, 0, 0, None, None) == -22
    assert lib.kvc_tp_exchange_max(fake, fake, fake, 2, 0, 1, 1, fake, fake, 1, 5, 1, None, None) == -22
    # IPC: NULL arguments are refused before any CUDA call
    handle = (ctypes.c_char * N.IPC_HANDLE_BYTES)()
    off = ctypes.c_int64()
    assert lib.kvc_ipc_export(0, None, handle, ctypes.byref(off)) == -14
    assert lib.kvc_ipc_open(0, None, ctypes.byref(ctypes.c_void_p())) == -14
    assert lib.kvc_ipc_close(0, None) == -14
    # un-rotation: NULL, unknown dtype, odd rotary dim, rotary dim above head dim, short rows
    assert lib.kvc_unrotate_queries(None, 0, 4, 128, 1, 128, 128, 0, fake, None) == -14
    assert lib.kvc_unrotate_queries(fake, 7, 4, 128, 1, 128, 128, 0, fake, None) == -22
    assert lib.kvc_unrotate_queries(fake, 0, 4, 128, 1, 128, 63, 0, fake, None) == -22
    assert lib.kvc_unrotate_queries(fake, 0, 4, 128, 1, 64, 128, 0, fake, None) == -22
    assert lib.kvc_unrotate_queries(fake, 0, 4, 100, 1, 128, 128, 0, fake, None) == -22
    # head statistics: more query heads than one CTA covers
    assert lib.kvc_head_stats(fake, 1, 1, 1, 4, 1025, fake, fake, fake, fake, fake, None) == -95


def test_host_helpers_validate_without_cuda_calls():
    lib = N.lib()
    fake = ctypes.c_void_p(0x1000)
    assert lib.kvc_record_event(None, None) == -14
    assert lib.kvc_copy_async(None, fake, 4, None) == -14
    assert lib.kvc_copy_async(fake, fake, -1, None) == -22
    assert lib.kvc_copy_async(fake, fake, 0, None) == 0  # nothing to copy, nothing launched


def test_header_compiles_as_c_and_links(tmp_path):
    """include/kvc.h is a C header: a C11 program includes it, links the library and agrees on the
    step descriptor's size and the offset of its last field (ctypes mirror included)."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "t.c"
    src.write_text(
        "#include <stddef.h>\n#include <stdio.h>\n#include \"kvc.h\"\n"
        "int main(void) {\n"
        "  printf(\"%d %lld %zu\\n\", kvc_abi_version(), (long long)kvc_triattention_step_size(),\n"
        "         offsetof(kvc_triattention_step, epoch));\n"
        "  return 0;\n}\n")
    libdir = N.library_path().parent
    exe = tmp_path / "t"
    r = subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-pedantic", f"-I{HEADER.parent}", str(src),
                        f"-L{libdir}", "-lkvc_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert int(out[0]) == N.ABI_VERSION
    assert int(out[1]) == ctypes.sizeof(N.TriAttentionStep)
    assert int(out[2]) == N.TriAttentionStep.epoch.offset
