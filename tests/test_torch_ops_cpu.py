"""torch.ops.murmurative_attention on the CPU: the reference's seven schemas are registered
verbatim (torch-ext/torch_binding.cpp:6-33), the north-star operator and its forward/backward
parts exist, and the fake (meta) implementations give the shapes, dtypes and layouts the CUDA
kernels produce, so FakeTensor tracing works without a GPU."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import murmurative_attention_b200  # noqa: F401  (registers the operators)
from murmurative_attention_b200 import torch_ops

NS = torch.ops.murmurative_attention


def _norm(schema: str) -> str:
    return " ".join(schema.replace("murmurative_attention::", "").split())


def test_reference_schemas_registered_verbatim():
    for name, schema in torch_ops.REFERENCE_SCHEMAS.items():
        assert _norm(str(getattr(NS, name).default._schema)) == _norm(schema), name
    for name in torch_ops.NORTH_STAR_SCHEMAS:
        assert hasattr(NS, name)


def test_fake_shapes_of_every_operator():
    with FakeTensorMode():
        B, H, N, M, D = 2, 3, 130, 64, 64
        q = torch.empty(B, N, H, D, dtype=torch.float16, device="cuda").transpose(1, 2)  # projection layout
        sk = torch.empty(B, H, M, D, dtype=torch.float16, device="cuda")
        out, idx, w = NS.slot_murmurate(q, sk, sk)
        assert out.shape == q.shape and out.stride() == q.stride() and out.dtype == q.dtype
        assert idx.shape == (B, H, N, 7) and idx.dtype == torch.int64 and w.dtype == torch.float32
        o, ww, ii = NS.slot_select_attend(q, sk, sk, None, True, None, None, M)
        assert o.shape == q.shape and ww.dtype == torch.float32 and ii.dtype == torch.int64
        gq, gk, gv = NS.slot_select_attend_backward(o, ww, q, sk, sk, ii, ww, None)
        assert gq.shape == q.shape and gk.shape == sk.shape
        r = NS.slot_update_backward(sk, sk, q, q, ii, ww, 0.9)
        assert [t.shape for t in r] == [q.shape, q.shape, sk.shape, sk.shape, (B, H, N, 7)]
        dk, dv = NS.slot_diffusion_backward(sk, sk, 0.15)
        assert dk.shape == sk.shape
        o4 = NS.slot_murmurate_fwd(q, sk, sk, 3, 7, False, 0.9, 0.15, None)
        assert o4[3].dtype == torch.uint8 and o4[3].dim() == 1 and o4[3].numel() > 0
        g3 = NS.slot_murmurate_bwd(out, w, q, o4[3], M, 3, 7, False, 0.9, 0.15, None)
        assert g3[0].shape == q.shape and g3[1].shape == sk.shape
