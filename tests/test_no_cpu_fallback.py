"""CPU: the product path has no CPU fallback -- the public calls given CPU
tensors raise a Bq4Error instead of computing anything."""
import pytest
import torch

from burn_image_b200 import f16 as F
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error


def test_q_matmul_refuses_cpu_tensors():
    K, N = 256, 128
    qt = q4.QuantizedTensor(torch.zeros((K // 8, N), dtype=torch.int32), torch.ones((K // 128, N)), (K, N),
                            q4.QuantScheme(store_packed_dim=0, level=(128,)))
    with pytest.raises(Bq4Error, match="GPU only"):
        q4.q_matmul(torch.zeros((4, K)), qt)


def test_packed_f16_and_attention_refuse_cpu_tensors():
    with pytest.raises(Bq4Error, match="CUDA tensor"):
        F.packed_f16_rhs_matmul(torch.zeros((4, 64)), torch.zeros((64, 32)).half())
    q = torch.zeros((1, 2, 8, 128)).half()
    with pytest.raises(Bq4Error, match="CUDA tensor"):
        F.attention(q, q, q)
