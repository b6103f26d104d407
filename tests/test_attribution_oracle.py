"""The oracle's restatement of src/attribution.rs:49-123 against the reference's
own attribution test (src/attribution.rs:246-263): credits sum to the finite loss
change, the credit of the row the edit lowered is negative, and restored_loss of
the changed row equals the loss of the restored logits.  No GPU."""
import numpy as np


def test_reference_attribution_example(oracle):
    before = np.array([[3.0, -1.0, 0.0]], np.float32)
    after = np.array([[0.0, 2.0, 1.0]], np.float32)
    c, g = oracle.integrated_credits(before, after, [1], [1.0], 128, gradients=True)
    expected = oracle.loss(before[0], 1) - oracle.loss(after[0], 1)
    assert abs(c.sum() - expected) < 1e-8
    assert c[2] < 0
    assert abs(oracle.restored_loss(after[0], 1, -1.0, 1) - oracle.loss(np.array([0.0, -1.0, 1.0], np.float32), 1)) < 1e-14
    # the integral of (softmax - onehot) sums to zero over the vocabulary
    assert abs(g.sum()) < 1e-12
