"""Model-level smoke of the hot path inside transformers' own model code:
the BERT-base fine-tune step with compressed FFN layers (CUDA8BitAdam) and a
small Llama-shaped decoder with every Linear compressed (ShardedAdam8), as
the bench's bert / llama8b workloads build them, at reduced depth.  The loss
on a fixed batch must be finite and fall."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(model, opt, batch_fn, steps):
    losses = []
    for _ in range(steps):
        opt.zero_grad(set_to_none=True)
        loss = batch_fn()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


def test_bert_finetune_steps(cuda):
    from packr_b200 import workloads as wl
    from packr_b200.cuda_adam import CUDA8BitAdam
    dev = torch.device("cuda")
    model = wl.bert_classifier(dev, layers=2, seed=0)
    packr = [m for m in model.modules() if m.__class__.__name__ == "PackRLinear"]
    assert len(packr) == 4
    model.eval()  # no dropout: the loss on the fixed batch must fall step by step
    opt = CUDA8BitAdam([p for p in model.parameters() if p.requires_grad], lr=2e-4)
    ids, labels = wl.bert_batch(dev, batch=8, seq=64)
    before = packr[0].W_f.detach().clone()
    losses = _train(model, opt, lambda: model(input_ids=ids, labels=labels).loss, 6)
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
    assert not torch.equal(before, packr[0].W_f.detach())


def test_llama_decoder_steps(cuda):
    from packr_b200 import workloads as wl
    from packr_b200.dp import ShardedAdam8
    dev = torch.device("cuda")
    model = wl.llama_decoder(dev, layers=2, seed=0, hidden_size=256, intermediate_size=512,
                             num_attention_heads=4, num_key_value_heads=2, vocab_size=1024)
    wrapped = [m for m in model.modules() if m.__class__.__name__ == "_Cast"]
    assert len(wrapped) == 2 * 7 + 1  # q k v o gate up down per layer, and lm_head
    assert not any(isinstance(m, torch.nn.Linear) for m in model.modules())
    model.eval()
    opt = ShardedAdam8([p for p in model.parameters() if p.requires_grad], lr=1e-3)
    ids = wl.llama_batch(dev, seq=128, vocab=1024)
    losses = _train(model, opt, lambda: model(input_ids=ids, labels=ids).loss, 6)
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
