"""The C-ABI library loads and exports every entry point include/gmoe.h
declares (CPU only: no compute calls)."""
import ctypes
import os
import re

import gmoe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gmoe.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gm_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_surface():
    names = declared_functions()
    for must in ("gm_moe_create", "gm_moe_forward", "gm_moe_forward_sync", "gm_router_select",
                 "gm_build_expert_schedules", "gm_bq_phase1_gate_up", "gm_bq_phase2_down",
                 "gm_combine"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(gmoe.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_functions()) == set(gmoe.SIGNATURES)


def test_version_and_error_text_without_gpu():
    L = gmoe.lib()
    assert b"sm_100a" in L.gm_version()
    assert L.gm_last_error(None) is not None


def test_create_rejects_bad_arguments():
    L = gmoe.lib()
    h = ctypes.c_void_p()
    assert L.gm_moe_create(ctypes.byref(h), 0, 0, 1, 0, 1) == -1          # max_tokens
    assert L.gm_moe_create(ctypes.byref(h), 0, 16, 1, 0, 3) == -1         # degree ∤ 128
    assert L.gm_moe_create(ctypes.byref(h), 0, 16, 1, 2, 2) == -1         # rank >= degree
    assert b"degree" in L.gm_last_error(None)


def test_workspace_size_grows_with_tokens():
    L = gmoe.lib()
    a, b = L.gm_moe_workspace_bytes(16), L.gm_moe_workspace_bytes(1024)
    assert 0 < a < b
    assert L.gm_moe_workspace_bytes(0) == 0


def test_stage_stat_layout_matches_header(tmp_path):
    """gmoe.StageStat mirrors gm_stage_stat_t byte for byte (checked by
    compiling the header with the host C compiler)."""
    import subprocess
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "gmoe.h"\n'
        'int main(void) { printf("%zu %zu %zu %zu %zu %zu %zu\\n", sizeof(gm_stage_stat_t),'
        ' offsetof(gm_stage_stat_t, label), offsetof(gm_stage_stat_t, calls),'
        ' offsetof(gm_stage_stat_t, kernels), offsetof(gm_stage_stat_t, total_ms),'
        ' offsetof(gm_stage_stat_t, min_ms), offsetof(gm_stage_stat_t, max_ms)); return 0; }\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    S = gmoe.StageStat
    want = [ctypes.sizeof(S)] + [getattr(S, f).offset for f in
                                 ("label", "calls", "kernels", "total_ms", "min_ms", "max_ms")]
    assert got == want


def test_profile_read_rejects_null_handle():
    L = gmoe.lib()
    n, k = ctypes.c_int(0), ctypes.c_long(0)
    assert L.gm_moe_profile_read(None, None, 0, ctypes.byref(n), ctypes.byref(k)) == -1


def test_attention_entry_points_validate_before_any_launch():
    """Geometry and sharding checks of the stateless attention calls run on
    the host before any CUDA call, so they answer without a GPU."""
    L = gmoe.lib()
    z = ctypes.c_void_p(0)

    def decode(head_dim=256, num_q=16, num_kv=8, window=1024, degree=1, rank=0, T=1):
        return L.gm_bq_attention_decode(z, z, z, z, z, z, z, z, T, head_dim, num_q, num_kv, window,
                                        degree, rank, 6, 63, 1, 1024, z, z, ctypes.c_size_t(0), z)

    assert decode(head_dim=128) == -1 and b"head_dim" in L.gm_last_error(None)
    assert decode(num_q=12, num_kv=8) == -1 and b"num_q" in L.gm_last_error(None)
    assert decode(degree=2, rank=1) == -1 and b"cache_degree" in L.gm_last_error(None)
    assert decode(window=0, degree=2, rank=0) == -1 and b"cache_degree" in L.gm_last_error(None)
    assert decode(T=1) == -1 and b"workspace" in L.gm_last_error(None)
    assert L.gm_bq_attention_workspace_bytes(0, 256, 16, 8, 1024) == 0
    assert L.gm_bq_attn_prep(z, z, z, z, z, z, z, z, z, z, z, z, z, z, z, 1, z, 1, 512, 16, 2, 128,
                             128, 1, 0, 6, 63, -1, z) == -1
    assert b"geometry" in L.gm_last_error(None)


def test_norm_residual_add_validates_before_any_launch():
    """gm_norm_residual_add rejects NULL, negative T and buffers that are not
    16-byte aligned on the host (no address is read), and T = 0 is a no-op."""
    L = gmoe.lib()
    p = ctypes.c_void_p
    assert L.gm_norm_residual_add(p(0), p(256), p(256), 1, p(256), p(0)) == -1
    assert b"NULL" in L.gm_last_error(None)
    assert L.gm_norm_residual_add(p(256), p(256), p(256), -1, p(256), p(0)) == -1
    assert L.gm_norm_residual_add(p(256), p(258), p(256), 1, p(256), p(0)) == -1
    assert b"16-byte" in L.gm_last_error(None)
    assert L.gm_norm_residual_add(p(0), p(0), p(0), 0, p(0), p(0)) == 0


def test_header_compiles_as_c_and_cxx_and_links(tmp_path):
    """A C99 consumer (what Mojo's external_call, cgo or a ctypes user sees):
    the header compiles warning-free as C99 and C++17, every declared entry
    point links from libgmoe.so, and host-only calls answer without a GPU."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        import pytest
        pytest.skip("no C compiler")
    names = declared_functions()
    table = ",\n    ".join("(fn)%s" % n for n in names)
    src = tmp_path / "consumer.c"
    src.write_text('''#include "gmoe.h"
#include <stdio.h>
#include <string.h>
typedef void (*fn)(void);
static fn every_entry_point[] = {
    %s
};
int main(void) {
  gm_moe_t* h = NULL;
  const char* v = gm_version();
  if (!v || !strstr(v, "sm_100a")) return 1;
  if (gm_moe_workspace_bytes(0) != 0) return 2;
  if (gm_moe_create(&h, 0, 0, 1, 0, 1) != GM_EINVAL || h != NULL) return 3;
  if (!strstr(gm_last_error(NULL), "max_tokens")) return 4;
  printf("%%s %%d\\n", v, (int)(sizeof every_entry_point / sizeof every_entry_point[0]));
  return 0;
}
''' % table)
    inc = os.path.join(ROOT, "include")
    libdir = os.path.dirname(gmoe.LIB_PATH)
    exe = tmp_path / "consumer"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", inc, str(src), "-o", str(exe),
                    "-L", libdir, "-lgmoe", "-Wl,-rpath," + libdir], check=True)
    gxx = shutil.which("g++")
    if gxx:
        subprocess.run([gxx, "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", "c++",
                        "-I", inc, str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert "sm_100a" in " ".join(out) and int(out[-1]) == len(names)


def test_no_gpu_means_an_error_not_a_fallback():
    """Without a GPU the product path fails with a CUDA status and text; there
    is no CPU path behind it."""
    import pytest
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(gmoe.GmoeError, match="GM_ECUDA"):
        gmoe.MoeBlock(16, 1)
    h = ctypes.c_void_p()
    assert gmoe.lib().gm_moe_create(ctypes.byref(h), 0, 16, 1, 0, 1) == -2   # GM_ECUDA
    assert not h.value


def test_call_checks_the_argument_count():
    import pytest
    with pytest.raises(TypeError, match="takes 5 arguments, 4 given"):
        gmoe.call("gm_rms_norm", 0, 0, 1, 0)
    with pytest.raises(TypeError, match="takes 5 arguments, 6 given"):
        gmoe.call("gm_rms_norm", 0, 0, 1, 0, None, None)


def test_missing_library_raises(monkeypatch):
    """No libgmoe.so: the binding raises on first use (no fallback)."""
    import pytest
    monkeypatch.setattr(gmoe, "_LIB", None)
    monkeypatch.setattr(gmoe, "LIB_PATH", os.path.join(ROOT, "no-such-dir", "libgmoe.so"))
    with pytest.raises(gmoe.GmoeError, match="not built"):
        gmoe.lib()
    with pytest.raises(gmoe.GmoeError, match="not built"):
        gmoe.call("gm_rms_norm", 0, 0, 1, 0, None)
