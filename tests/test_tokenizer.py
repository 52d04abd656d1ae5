"""Tokenizer wrapper: EOS handling, truncation in both directions, config-driven construction."""
import pytest

from olmo_b200.config import ModelConfig, TokenizerConfig, TrainConfig
from olmo_b200.exceptions import OLMoConfigurationError
from olmo_b200.tokenizer import Tokenizer

tokenizers = pytest.importorskip("tokenizers")

WORDS = "the quick brown fox jumps over lazy dog and runs far away from here".split()


@pytest.fixture(scope="module")
def tok_file(tmp_path_factory):
    from tokenizers import Tokenizer as Base
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    vocab = {w: i for i, w in enumerate(WORDS)}
    vocab["<unk>"] = len(vocab)
    vocab["<eos>"] = len(vocab)
    base = Base(WordLevel(vocab, unk_token="<unk>"))
    base.pre_tokenizer = Whitespace()
    base.add_special_tokens(["<eos>"])
    path = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    base.save(str(path))
    return path, len(vocab)


def test_encode_decode_and_eos(tok_file):
    path, n = tok_file
    tok = Tokenizer.from_file(path)
    assert tok.vocab_size == n and tok.eos_token_id == n - 1 and tok.pad_token_id == n - 1
    ids = tok.encode("the quick brown fox")
    assert ids == [0, 1, 2, 3, n - 1]
    assert tok.encode("the quick", add_special_tokens=False) == [0, 1]
    assert tok.decode(ids) == "the quick brown fox"
    assert tok.eos_token == "<eos>" and tok.pad_token == "<eos>"
    # EOS is appended once, never doubled
    assert tok.add_special_tokens([0, n - 1]) == [0, n - 1]
    assert tok.add_special_tokens([]) == [n - 1]
    assert tok.num_special_tokens_to_add() == 1 and tok.num_special_tokens_to_add(is_pair=True) == 2


@pytest.mark.parametrize("direction,want", [("right", [0, 1, 2]), ("left", [4, 5, 6])])
def test_truncation(tok_file, direction, want):
    path, n = tok_file
    tok = Tokenizer.from_file(path, truncate_to=4, truncate_direction=direction)
    text = "the quick brown fox jumps over lazy"
    assert tok.encode(text) == want + [n - 1]
    assert tok.encode(text, add_special_tokens=False) == ([0, 1, 2, 3] if direction == "right" else [3, 4, 5, 6])
    assert tok.encode_batch(["the", text]) == [[0, n - 1], want + [n - 1]]


def test_from_train_config_and_checkpoint(tok_file, tmp_path):
    path, n = tok_file
    cfg = TrainConfig(
        model=ModelConfig(vocab_size=n, eos_token_id=n - 1, pad_token_id=n - 2),
        tokenizer=TokenizerConfig(identifier=str(path)),
    )
    tok = Tokenizer.from_train_config(cfg)
    assert tok.eos_token_id == n - 1 and tok.pad_token_id == n - 2
    cfg.save(tmp_path / "config.yaml")
    again = Tokenizer.from_checkpoint(tmp_path)
    assert again.encode("lazy dog") == tok.encode("lazy dog")
    cfg.model.vocab_size = n + 5
    with pytest.raises(OLMoConfigurationError):
        Tokenizer.from_train_config(cfg)


def test_packaged_lookup(tok_file, tmp_path, monkeypatch):
    path, n = tok_file
    root = tmp_path / "data"
    (root / "tokenizers").mkdir(parents=True)
    (root / "tokenizers" / "tiny.json").write_bytes(path.read_bytes())
    monkeypatch.setenv("OLMO_DATA_DIR", str(root))
    cfg = TrainConfig(model=ModelConfig(vocab_size=n, eos_token_id=n - 1), tokenizer=TokenizerConfig(identifier="tokenizers/tiny.json"))
    assert Tokenizer.from_train_config(cfg).vocab_size == n
    cfg.tokenizer.identifier = "tiny"
    assert Tokenizer.from_train_config(cfg).vocab_size == n
