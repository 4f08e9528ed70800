"""SuffixDecoding's suffix trie (counts, longest match, path and tree speculation) against brute force on token
lists, and lossless decoding with it on the CPU fp32 path."""

import random
from collections import Counter

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import ConfigError
from economize_b200.techniques.suffix_decoding import SuffixDecodingConfig, SuffixTrie, load_datastore

from .helpers import prompts, tiny_model


def _substring_counts(seqs, depth):
    counts = Counter()
    for s in seqs:
        for i in range(len(s)):
            for L in range(1, depth + 1):
                if i + L <= len(s):
                    counts[tuple(s[i:i + L])] += 1
    return counts


def test_counts_match_brute_force():
    rng = random.Random(0)
    seqs = [[rng.randrange(5) for _ in range(rng.randrange(5, 40))] for _ in range(4)]
    trie = SuffixTrie(6)
    for s in seqs[:2]:
        trie.add_sequence(s)
    trie.append(seqs[2][:10])  # incremental appends of one sequence
    trie.append(seqs[2][10:])
    trie.end_sequence()
    trie.add_sequence(seqs[3])
    want = _substring_counts(seqs, 6)

    def walk(node, prefix):
        for tok, child in trie.children[node].items():
            path = prefix + (tok,)
            assert trie.count[child] == want[path], path
            walk(child, path)
    walk(0, ())
    assert sum(1 for k in want) == len(trie) - 1  # every substring is exactly one node


def test_path_speculation_follows_the_most_frequent_continuation():
    trie = SuffixTrie(8)
    trie.add_sequence([7, 1, 2, 3, 9, 1, 2, 3, 9, 1, 2, 4])
    spec = trie.speculate([5, 1, 2], max_tokens=3, min_prob=0.1, tree=False, factor=2.0)
    # after (1, 2): 3 twice, 4 once -> 3 (p 2/3), then 9 (p 2/3 * 1), then 1 (p 2/3 * 1 * 1)
    assert spec.tokens == (3, 9, 1) and spec.parents == (-1, 0, 1) and spec.match == 2
    assert spec.score == pytest.approx(3 * 2 / 3)
    # the adaptive length: a 2-token match drafts at most floor(1.0 * 2) = 2 tokens
    assert trie.speculate([5, 1, 2], max_tokens=3, min_prob=0.1, tree=False).tokens == (3, 9)
    tree = trie.speculate([5, 1, 2], max_tokens=3, min_prob=0.3, tree=True, factor=2.0)
    assert tree.tokens[:2] == (3, 9) and set(tree.tokens) <= {3, 9, 4, 1}
    assert trie.speculate([5, 1, 2], max_tokens=2, min_prob=0.9, tree=False).tokens == ()


def test_adaptive_length_and_depth_limit():
    trie = SuffixTrie(4)
    trie.add_sequence([1, 2, 3, 4, 5, 6])
    # a 3-token match leaves room for depth - 3 = 1 more token, a 2-token match drafts 2: the better draft wins
    assert trie.speculate([1, 2, 3], max_tokens=8, min_prob=0.1, tree=False).tokens == (4, 5)
    assert trie.speculate([9, 2, 3], max_tokens=8, min_prob=0.1, tree=False).tokens == (4, 5)
    # factor 0.5: a 1-token match drafts floor(0.5) = 0 tokens; 2 tokens drafts 1
    assert trie.speculate([2], max_tokens=8, min_prob=0.1, tree=False, factor=0.5).tokens == ()
    assert trie.speculate([2, 3], max_tokens=8, min_prob=0.1, tree=False, factor=0.5).tokens == (4,)


def test_config_checks_and_datastore(tmp_path):
    with pytest.raises(ConfigError):
        SuffixDecodingConfig(max_depth=1)
    with pytest.raises(ConfigError):
        SuffixDecodingConfig(min_token_prob=0.0)
    path = tmp_path / "store.jsonl"
    path.write_text("[1, 2, 3]\n[4, 5]\n")
    assert load_datastore(str(path)) == [[1, 2, 3], [4, 5]]


@pytest.mark.parametrize("tree", [False, True])
def test_suffix_decoding_is_lossless_and_accepts_repeats(tree):
    model = tiny_model()
    plain = eco.apply(model).decode_batch(prompts(), 24, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, SuffixDecodingConfig(tree=tree, max_spec_tokens=6))
    em.techniques["suffix_decoding"].add_corpus([torch.cat([p, r.tokens]).tolist() for p, r in
                                                 zip(prompts(), plain)])
    out = em.decode_batch(prompts(), 24, decoding=eco.DecodeConfig(cycle_length=7))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)
    assert sum(r.accepted for r in out) > 0  # the global trie holds these very continuations
