"""The C-ABI library loads and exports every function include/krystal_cuda.h declares.

No compute call runs here (there may be no GPU); the GPU tests call through it.
"""
import re
from pathlib import Path

from krystal_b200 import abi

HEADER = Path(__file__).resolve().parent.parent / "include" / "krystal_cuda.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(kc_[a-z_]+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared_functions() == set(abi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.kc_abi_version() == 1


def test_struct_sizes_match_the_c_layout():
    import ctypes as C
    assert C.sizeof(abi.KcConfig) == 13 * 4 + 4 + 8 + 4 + 4  # 13 u32, pad, pointer, u32, tail pad
    assert C.sizeof(abi.KcBatchView) == 8 + 8 + 8 * 9 + 8 + 8
    assert C.sizeof(abi.KcBatchOut) == 8 * 11


STRUCTS = {"kc_config": "KcConfig", "kc_block_view": "KcBlockView", "kc_weights_view": "KcWeightsView",
           "kc_changes": "KcChanges", "kc_frame_view": "KcFrameView", "kc_encoded_view": "KcEncodedView",
           "kc_mask_rule": "KcMaskRule", "kc_batch_view": "KcBatchView", "kc_batch_out": "KcBatchOut",
           "kc_device_result": "KcDeviceResult", "kc_stage_times": "KcStageTimes",
           "kc_backward_out": "KcBackwardOut", "kc_backward_result": "KcBackwardResult",
           "kc_stream_result": "KcStreamResult", "kc_batch_select_view": "KcBatchSelectView",
           "kc_learn_options": "KcLearnOptions", "kc_stream_options": "KcStreamOptions",
           "kc_stream_stats": "KcStreamStats"}


def test_struct_layouts_match_the_header(tmp_path):
    """Every field offset of every ctypes struct equals the C compiler's, read
    from a probe compiled against include/krystal_cuda.h."""
    import ctypes as C
    import subprocess
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, pyname in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in getattr(abi, pyname)._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["return 0; }"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    want = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, f, v = line.split()
        want[(cname, f)] = int(v)
    for cname, pyname in STRUCTS.items():
        cls = getattr(abi, pyname)
        assert C.sizeof(cls) == want[(cname, "size")], cname
        for f, _ in cls._fields_:
            assert getattr(cls, f).offset == want[(cname, f)], (cname, f)
