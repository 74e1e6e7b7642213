# SPDX-License-Identifier: Apache-2.0
"""The seeded synthetic token stream that stands in for the tokenized story
corpus of the reference's LM A/B: deterministic, in range, with the
end-of-story rate and the bigram structure it is built with."""
import torch

import bench


def test_story_tokens_are_seeded_and_structured():
    a = bench.synthetic_story_tokens(60000, seed=3)
    b = bench.synthetic_story_tokens(60000, seed=3)
    c = bench.synthetic_story_tokens(60000, seed=4)
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert a.dtype == torch.int64 and int(a.min()) >= 0 and int(a.max()) < bench.GPT2_VOCAB
    eos = bench.GPT2_VOCAB - 1
    rate = float((a == eos).float().mean())
    assert 0.5 / 200 < rate < 2.0 / 200
    # a token's most frequent follower accounts for far more than its unigram share
    prev, nxt = a[:-1], a[1:]
    common = int(torch.mode(prev[prev != eos]).values)
    followers = nxt[prev == common]
    top = int(torch.mode(followers).values)
    assert float((followers == top).float().mean()) > 0.4
