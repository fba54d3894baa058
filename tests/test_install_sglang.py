"""CPU: the SGLang hook installer against a fake SGLang tree holding the three call sites.

The fake files carry the site text of SGLang 0.5.22 that the reference's installer matches
(patches/apply_sglang_fp8_hand_gemm.py:22-65); the installer must patch each exactly once, leave a patched
tree unchanged on a second run, refuse a tree whose site text differs without writing anything, and the
patched GEMM entry must call the drop-in module's `matmul` before its own (Triton) path.
"""
import sys
import types

import pytest

FP8_KERNEL = '''import torch
from sglang.srt.layers import deep_gemm_wrapper


def prepare_block_fp8_matmul_inputs(A, B, As, Bs, block_size, output_dtype):
    M = A.numel() // A.shape[-1]
    N, K = B.shape
    C = A.new_empty(A.shape[:-1] + (N,), dtype=output_dtype)
    return M, N, K, C


def w8a8_block_fp8_matmul_triton(A, B, As, Bs, block_size, output_dtype=torch.float16):
    M, N, K, C = prepare_block_fp8_matmul_inputs(A, B, As, Bs, block_size, output_dtype)

    block_n, block_k = block_size
    C.fill_(-1)
    return C
'''

QWEN2_MOE = '''class Qwen2MoeMLP:
    def forward(
        self,
        x,
    ):
        gate_up, _ = self.gate_up_proj(x)
        if self._enable_silu_fp4_quant_fusion and not isinstance(gate_up, tuple):
            pass
        return gate_up
'''

LOADER = '''def load_weights_and_postprocess(model, weights, target_device):
    if True:
        maybe_quantize_lm_head(model)
    return model
'''


def _tree(root):
    (root / "kernels/ops/gemm").mkdir(parents=True)
    (root / "srt/models").mkdir(parents=True)
    (root / "srt/model_loader").mkdir(parents=True)
    (root / "kernels/ops/gemm/fp8_kernel.py").write_text(FP8_KERNEL)
    (root / "srt/models/qwen2_moe.py").write_text(QWEN2_MOE)
    (root / "srt/model_loader/loader.py").write_text(LOADER)
    return root


def test_installer_patches_each_site_once(tmp_path):
    from fp8_hand_b200 import install_sglang as inst
    root = _tree(tmp_path / "sglang")
    logs = []
    res = inst.install(root, build=False, log=logs.append)
    assert set(res.values()) == {"patched"}
    gemm = (root / inst.GEMM_FILE).read_text()
    assert gemm.count("if fp8_hand_sm89.matmul(A, B, C, As, Bs, M, N, K, block_size):") == 1
    assert gemm.count(inst.MODULE_IMPORT) == 1
    mlp = (root / inst.MLP_FILE).read_text()
    assert "fused = fp8_hand_sm89.fused_gate_up(self.gate_up_proj, x)" in mlp
    loader = (root / inst.LOADER_FILE).read_text()
    assert "fp8_hand_sm89.relayout(model)" in loader
    for rel in (inst.GEMM_FILE, inst.MLP_FILE, inst.LOADER_FILE):
        compile((root / rel).read_text(), rel, "exec")  # still valid Python
    # a second run finds the marks and changes nothing
    before = {rel: (root / rel).read_text() for rel, _ in inst.SITES}
    assert set(inst.install(root, build=False, log=logs.append).values()) == {"already patched"}
    assert {rel: (root / rel).read_text() for rel, _ in inst.SITES} == before


def test_installer_refuses_unknown_site_text_without_writing(tmp_path):
    from fp8_hand_b200 import install_sglang as inst
    root = _tree(tmp_path / "sglang")
    (root / inst.LOADER_FILE).write_text(LOADER.replace("maybe_quantize_lm_head(model)", "quantize(model)"))
    before = {rel: (root / rel).read_text() for rel, _ in inst.SITES}
    with pytest.raises(inst.InstallError):
        inst.install(root, build=False, log=lambda *_: None)
    assert {rel: (root / rel).read_text() for rel, _ in inst.SITES} == before  # nothing half-patched
    assert inst.main(["--root", str(root), "--no-build"]) == 1


def test_patched_gemm_entry_calls_the_dropin_first(tmp_path, monkeypatch):
    """Execute the patched fp8_kernel.py with stub `sglang` imports: the hook returns the drop-in's C when
    matmul() takes the call, and falls through to the original path when it returns False."""
    import torch

    from fp8_hand_b200 import install_sglang as inst
    root = _tree(tmp_path / "sglang")
    inst.install(root, build=False, log=lambda *_: None)
    calls = []

    def fake_matmul(A, B, C, As, Bs, M, N, K, block_size):
        calls.append((M, N, K, tuple(block_size)))
        if getattr(B, "tiles", None) is None:
            return False
        C.fill_(7)
        return True

    mod = types.ModuleType("fp8_hand_b200.fp8_hand_sm100")
    mod.matmul = fake_matmul
    layers = types.ModuleType("sglang.srt.layers")
    layers.deep_gemm_wrapper = object()
    for name, m in {"sglang": types.ModuleType("sglang"), "sglang.srt": types.ModuleType("sglang.srt"),
                    "sglang.srt.layers": layers}.items():
        monkeypatch.setitem(sys.modules, name, m)
    pkg = sys.modules["fp8_hand_b200"]
    monkeypatch.setattr(pkg, "fp8_hand_sm100", mod, raising=False)
    monkeypatch.setitem(sys.modules, "fp8_hand_b200.fp8_hand_sm100", mod)
    ns = {}
    exec(compile((root / inst.GEMM_FILE).read_text(), "fp8_kernel.py", "exec"), ns)
    A = torch.zeros(3, 256)
    B = torch.zeros(128, 256)
    As, Bs = torch.ones(3, 2), torch.ones(1, 2)
    out = ns["w8a8_block_fp8_matmul_triton"](A, B, As, Bs, [128, 128], torch.float32)
    assert (out == -1).all() and calls[-1] == (3, 128, 256, (128, 128))  # no tiles: the original path
    B.tiles = object()
    out = ns["w8a8_block_fp8_matmul_triton"](A, B, As, Bs, [128, 128], torch.float32)
    assert (out == 7).all()  # the drop-in wrote C and the hook returned it
