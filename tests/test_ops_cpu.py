"""torch.ops.qhtp.*: every op is registered, and its fake implementation gives the output shape and
dtype without a GPU (FakeTensorMode), so models that use them can be traced on any host."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import qcom_htp_b200  # noqa: F401  (registers the ops)

OPS = ["matmul_u8i8", "matmul_w4a8", "matmul_w8a16", "matmul_w4a16", "matmul_w16a16",
       "matmul_per_group_w4a8", "matmul_per_group_w4a16",
       "gdn_inverse", "gdn_chunk_inverse", "gdn_solve_u16"]


def test_all_ops_registered():
    for name in OPS:
        assert hasattr(torch.ops.qhtp, name), name


def test_fake_shapes():
    with FakeTensorMode():
        d = "cuda"
        f32 = lambda *s: torch.empty(s, device=d)
        i32 = lambda *s: torch.empty(s, dtype=torch.int32, device=d)
        a8 = torch.empty((5, 64), dtype=torch.uint8, device=d)
        a16 = torch.empty((5, 64), dtype=torch.uint16, device=d)
        out = torch.ops.qhtp.matmul_u8i8(a8, torch.empty((96, 64), dtype=torch.int8, device=d), f32(96), i32(96),
                                         None, 0, 0.1, -128, 0.2, 0)
        assert out.shape == (5, 96) and out.dtype == torch.uint8
        out = torch.ops.qhtp.matmul_w4a16(a16, torch.empty((32, 96), dtype=torch.uint8, device=d), f32(96),
                                          i32(96), torch.empty((96, 1), dtype=torch.uint8, device=d), 64, 0.1,
                                          -32768, 0.2, -32768)
        assert out.shape == (5, 96) and out.dtype == torch.uint16
        out = torch.ops.qhtp.matmul_w16a16(a16, torch.empty((96, 64), dtype=torch.int16, device=d), f32(96),
                                           i32(96), None, 0, 0.1, -32768, 0.2, -32768)
        assert out.shape == (5, 96) and out.dtype == torch.uint16
        out = torch.ops.qhtp.matmul_per_group_w4a16(a16, torch.empty((32, 96), dtype=torch.uint8, device=d),
                                                    f32(96, 1), f32(96), 0.1, -32768, 0.2, -32768)
        assert out.shape == (5, 96) and out.dtype == torch.uint16
        out = torch.ops.qhtp.matmul_per_group_w4a8(a8, torch.empty((32, 96), dtype=torch.uint8, device=d),
                                                   f32(96, 1), f32(96), 0.1, -128, 0.2, 0)
        assert out.shape == (5, 96) and out.dtype == torch.uint8
        A = torch.empty((3, 256, 256), dtype=torch.bfloat16, device=d)
        assert torch.ops.qhtp.gdn_inverse(A).dtype == torch.float32
        Ac = torch.empty((3, 64, 64), dtype=torch.uint16, device=d)
        assert torch.ops.qhtp.gdn_solve_u16(Ac, 32768, 1e-4, 32768, 1e-4).shape == (3, 64, 64)
        k = torch.empty((2, 3, 256, 128), dtype=torch.bfloat16, device=d)
        T = torch.ops.qhtp.gdn_chunk_inverse(k, f32(2, 3, 256), f32(2, 3, 256))
        assert T.shape == (2, 3, 256, 256) and T.dtype == torch.float32
