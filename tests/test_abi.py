"""The C-ABI library loads, exports every function include/*.h declares, and
its ctypes struct mirrors match the C layout (no GPU needed)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"

DECL = re.compile(r"^\s*(?:[A-Za-z_][\w\s\*]*?[\s\*])([A-Za-z_]\w*)\s*\(([^;{]*)\)\s*;", re.M)


def declared_functions() -> set[str]:
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//.*", "", text)
        text = re.sub(r"#.*", "", text)
        for m in DECL.finditer(text):
            names.add(m.group(1))
    return names


def test_headers_declare_the_reference_entry_points():
    names = declared_functions()
    # CrossCache include/cache/cache.h:8-23 and include/inner_h/device.h:43-50
    ref = {"cache_register", "cache_unregister", "cache_lookup", "cache_store", "cache_load",
           "cache_init", "cache_exit", "alloc_pinned_ptr", "free_pinned_ptr", "wrapper_ptr",
           "unwrapper_ptr", "open_ipc_keys", "close_ipc_keys", "transfer_kvcache", "reset_device"}
    assert ref <= names, ref - names
    assert {"cuda_adaptor_create", "cuda_adaptor_destroy", "kv_copy_launch",
            "kv_block_hash_launch", "transfer_kvcache_batch", "cache_lookup_batch"} <= names


def test_library_exports_every_declared_symbol():
    from demo_b200 import _lib

    lib = C.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    # every declared function has a ctypes signature in the bindings
    assert declared_functions() <= set(_lib.SIGNATURES), declared_functions() - set(_lib.SIGNATURES)


LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "inner.h"
#include "device.h"
#include "kvcopy.h"
#include "cache.h"
#define F(s, f) printf(#s "." #f " %zu\n", offsetof(struct s, f))
#define S(s) printf(#s " %zu\n", sizeof(struct s))
int main(void) {
  S(worker_context); F(worker_context, node_id); F(worker_context, per_token_size);
  F(worker_context, per_len); F(worker_context, k_raw_ptrs); F(worker_context, v_ptrs);
  S(model_info); F(model_info, hidden_dim_size);
  S(transfer_params); F(transfer_params, page_buffer_size); F(transfer_params, devid);
  F(transfer_params, num_layers); F(transfer_params, hidden_dim_size); F(transfer_params, direction);
  S(transfer_batch); F(transfer_batch, records); F(transfer_batch, num_records);
  F(transfer_batch, num_layers); F(transfer_batch, direction);
  F(transfer_batch, block_stride); F(transfer_batch, head_bytes);
  S(kv_copy_desc); F(kv_copy_desc, page_buffer_size); F(kv_copy_desc, direction); F(kv_copy_desc, flags);
  F(kv_copy_desc, layer_begin); F(kv_copy_desc, record_layers); F(kv_copy_desc, max_ctas);
  F(kv_copy_desc, block_stride); F(kv_copy_desc, head_bytes);
  S(cache_stats);
  return 0;
}
"""


def test_struct_layout_matches_ctypes(tmp_path):
    from demo_b200 import _lib

    src = tmp_path / "probe.c"
    src.write_text(LAYOUT_PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{INCLUDE}", str(src), "-o", str(exe)], check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True,
                                                               text=True, check=True).stdout.split("\n") if line)
    mirrors = {"worker_context": _lib.WorkerContext, "model_info": _lib.ModelInfo,
               "transfer_params": _lib.TransferParams, "transfer_batch": _lib.TransferBatch,
               "kv_copy_desc": _lib.KvCopyDesc, "cache_stats": _lib.CacheStats}
    for key, val in out.items():
        if "." in key:
            s, f = key.split(".")
            assert getattr(mirrors[s], f).offset == int(val), key
        else:
            assert C.sizeof(mirrors[key]) == int(val), key


def test_reference_struct_layout_unchanged(tmp_path):
    """worker_context / transfer_params are laid out exactly like the
    reference headers (compiled against CrossCache's own include/inner_h)."""
    from oracle import reference_root
    ref_inc = reference_root() / "include" / "inner_h"
    if not ref_inc.exists():
        pytest.skip("reference tree not present")
    probe = r"""
#include <stdio.h>
#include <stddef.h>
#include "inner.h"
#include "device.h"
int main(void){printf("%zu %zu %zu %zu %zu %zu\n", sizeof(struct worker_context),
 offsetof(struct worker_context, per_len), offsetof(struct worker_context, v_ptrs),
 sizeof(struct transfer_params), offsetof(struct transfer_params, hidden_dim_size),
 offsetof(struct transfer_params, direction));return 0;}
"""
    res = []
    for inc in (ref_inc, INCLUDE):
        src = tmp_path / "p.c"
        src.write_text(probe)
        exe = tmp_path / "p"
        subprocess.run(["gcc", "-std=gnu11", f"-I{inc}", str(src), "-o", str(exe)], check=True)
        res.append(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert res[0] == res[1]
