"""The whole-decoder handle (hxb_model_*) on the host side: the container's attention keys are read,
an MLA container is refused (the GPU path covers GQA / MHA; the reference binding keeps such a
model's attention on the CPU), a broken file is refused, and without a GPU the open fails instead of
falling back to the CPU."""
import os

import pytest

import hearth_b200 as hb

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except ImportError:
        return False


def test_mla_container_is_refused():
    with pytest.raises(RuntimeError, match="MLA"):
        hb.Model(os.path.join(GOLDEN, "tiny_deepseek_v3.hearth"))


def test_broken_container_is_refused(tmp_path):
    p = tmp_path / "broken.hearth"
    p.write_bytes(b"HRTH" + b"\0" * 100)
    with pytest.raises(RuntimeError):
        hb.Model(str(p))


@pytest.mark.parametrize("name", ["tiny_qwen3_moe", "tiny_olmoe", "tiny_mixtral", "tiny_qwen2_moe", "tiny_moe"])
def test_without_a_gpu_the_open_fails(name):
    if _has_gpu():
        pytest.skip("a GPU is present: tests/test_gpu_model.py covers the handle")
    with pytest.raises(RuntimeError, match="no such CUDA device"):
        hb.Model(os.path.join(GOLDEN, name + ".hearth"))
