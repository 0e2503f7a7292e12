"""The Python drop-in (CPU only): signature, backend validation, dtype rules,
and that it refuses to run anywhere but on CUDA tensors (no CPU fallback)."""
import importlib
import inspect

import pytest
import torch

import in_context_sparse_attention as ica
from oracle import icsa_oracle as orc

# the module (the package attribute of the same name is the function)
esa_mod = importlib.import_module("in_context_sparse_attention.editing_sparse_attention")


def test_exports_mirror_the_reference_package():
    reference = {"Backend", "editing_sparse_attention", "editing_sparse_attention_tilelang"}
    # plus the timeout reporting of this build (no counterpart in the reference)
    assert set(ica.__all__) == reference | {"IcsaError", "device_status"}
    assert ica.editing_sparse_attention_tilelang is ica.editing_sparse_attention


class _FakeLib:
    """Stands in for libicsa.so: returns fixed status codes (no GPU)."""

    def __init__(self, sticky, word):
        self.sticky, self.word, self.calls = sticky, word, []

    def icsa_last_status(self, stream, clear):
        self.calls.append(("last", stream, clear))
        return self.sticky

    def icsa_device_status(self, ws, stream):
        self.calls.append(("word", ws, stream))
        return self.word

    def icsa_last_error(self):
        return b"a device-side wait gave up (code 0x102)"


@pytest.mark.parametrize("sticky,word", [(5, 0), (0, 5)])
def test_status_check_raises_on_a_recorded_timeout(monkeypatch, sticky, word):
    fake = _FakeLib(sticky, word)
    monkeypatch.setattr(ica._capi, "load", lambda path=None: fake)
    with pytest.raises(ica.IcsaError) as e:
        esa_mod._check_status(fake, 1234, 7, "call")
    assert e.value.code == 5 and "ICSA_ERR_DEVICE_TIMEOUT" in str(e.value)
    assert fake.calls[0] == ("last", 7, 1)  # the per-device record is read and cleared first


def test_status_check_passes_when_clean(monkeypatch):
    fake = _FakeLib(0, 0)
    monkeypatch.setattr(ica._capi, "load", lambda path=None: fake)
    esa_mod._check_status(fake, 1234, 7, "call")
    assert fake.calls == [("last", 7, 1), ("word", 1234, 7)]


def test_signature_keeps_the_reference_parameters():
    params = list(inspect.signature(ica.editing_sparse_attention).parameters)
    assert params[:9] == ["q", "k", "v", "t_seq_len", "s_seq_len", "alpha_2", "alpha_3", "SPARSITY_RATIO", "backend"]
    sig = inspect.signature(ica.editing_sparse_attention)
    assert sig.parameters["alpha_2"].default == 1.0
    assert sig.parameters["SPARSITY_RATIO"].default == 0.0625


def test_backend_names():
    for name in ("b200", "tilelang", "triton"):
        assert ica.Backend.validate(name) == name
    with pytest.raises(ValueError, match="Unknown backend"):
        ica.Backend.validate("flash")


def test_cpu_tensors_are_refused():
    q = torch.randn(1, 128, 2, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ica.editing_sparse_attention(q, q, q, 64, 64)
    with pytest.raises(ValueError):
        ica.editing_sparse_attention(q, q, q, 64, 64, backend="flash")


@pytest.mark.parametrize("dts,alpha", [
    ((torch.bfloat16,) * 3, 1.0),
    ((torch.float32,) * 3, 1.0),
    ((torch.float32, torch.float32, torch.bfloat16), torch.zeros(1, 8, 1, 1)),
    ((torch.bfloat16,) * 3, torch.zeros(1, 8, 1, 1)),
    ((torch.bfloat16,) * 3, torch.zeros(1, 8, 1, 1, dtype=torch.bfloat16)),
])
def test_result_dtypes_follow_torch_promotion(dts, alpha):
    """Same rules as the reference's `x + out_compress * alpha_2` (with the
    compressed matmuls in bf16 whenever an input is bf16)."""
    got = esa_mod._result_dtypes(*dts, alpha)
    want = orc.result_dtypes(*dts, alpha)
    assert got == want
    q = torch.zeros(1, 8, 1, 4, dtype=dts[0])
    outc = torch.zeros(1, 8, 1, 4, dtype=want[0])
    assert (q + outc * alpha).dtype == want[2]


def test_default_head_groups_divide_and_stay_small():
    """Head groups for host streaming: a divisor of H, about eight groups,
    at least four heads per group when H allows."""
    for H, want in ((40, 5), (20, 4), (10, 2), (5, 1), (64, 8), (2, 2), (3, 3), (7, 1)):
        g = esa_mod._default_group_heads(H)
        assert H % g == 0 and g == want, (H, g)
