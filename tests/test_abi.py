"""The C-ABI libraries load on any machine (no GPU needed) and export every
function declared in include/*.h."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "qwen3-tts_b200", "lib")


def declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", src)
    skip = {"if", "sizeof", "defined", "extern"}
    return sorted({n for n in names if n.startswith(("qtb_", "qwen_cuda_")) and n not in skip})


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_engine_library_exports_everything_declared():
    syms = exported(os.path.join(LIB, "libqwen3tts_b200.so"))
    dropin = exported(os.path.join(LIB, "libqwen_tts_cuda_b200.so"))
    want = declared("qwen3tts_b200.h") + declared("qwen_tts_cuda_b200.h")
    missing = [n for n in want if n not in syms and n not in dropin]
    assert not missing, missing


def test_dropin_surface_matches_reference_names():
    # the reference's extern "C" surface of qwen_tts_cuda_talker.cu
    ref = ["qwen_cuda_talker_init", "qwen_cuda_talker_step", "qwen_cuda_talker_get_dec_x",
           "qwen_cuda_talker_upload_kv", "qwen_cuda_talker_free", "qwen_cuda_talker_batch_init",
           "qwen_cuda_talker_batch_step", "qwen_cuda_talker_batch_upload_slot", "qwen_cuda_talker_batch_free",
           "qwen_cuda_cp_init", "qwen_cuda_cp_step", "qwen_cuda_cp_free", "qwen_cuda_cp_batch_init",
           "qwen_cuda_cp_batch_step", "qwen_cuda_cp_batch_free", "qwen_cuda_batch_selftest"]
    syms = exported(os.path.join(LIB, "libqwen3tts_b200.so")) | exported(os.path.join(LIB, "libqwen_tts_cuda_b200.so"))
    assert [n for n in ref if n not in syms] == []


def test_library_loads_without_gpu():
    import qtts_b200 as Q
    L = Q.lib()
    assert L.qtb_device_count() >= 0
    assert isinstance(L.qtb_last_error(), bytes)


def test_engine_rejects_bad_device():
    import ctypes as C
    import qtts_b200 as Q
    d = Q.EngineDesc()
    h = C.c_void_p()
    rc = Q.lib().qtb_engine_create(C.byref(d), 99, C.byref(h))
    assert rc != 0 and not h.value
