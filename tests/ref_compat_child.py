"""Child process of ``test_reference_compat.py``: imports the *reference* package from ``baseline/_ref`` (never this
repository's), builds its model from a JSON model config, loads an unsharded ``model.pt`` written by this framework and
prints the logits for fixed token ids as JSON."""
import json
import sys
from pathlib import Path

root = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(root / "baseline" / "_ref"))
sys.path.insert(0, str(root / "baseline" / "shims"))

import torch  # noqa: E402
from olmo.config import ModelConfig  # noqa: E402  (the reference's)
from olmo.model import OLMo  # noqa: E402

cfg_json, ckpt, ids_json = sys.argv[1:4]
fields = json.loads(Path(cfg_json).read_text())
known = set(ModelConfig.__dataclass_fields__)
cfg = ModelConfig(**{k: v for k, v in fields.items() if k in known})
cfg.init_device = "cpu"
model = OLMo(cfg, init_params=False)
state = torch.load(Path(ckpt) / "model.pt", map_location="cpu", weights_only=False)
fixed, _ = model._make_state_dict_compatible(state)
missing, unexpected = model.load_state_dict(fixed, strict=True), None
model.eval()
ids = torch.tensor(json.loads(Path(ids_json).read_text()))
with torch.no_grad():
    logits = model(ids).logits
trainer = torch.load(Path(ckpt) / "train.pt", map_location="cpu", weights_only=False)
optim = torch.load(Path(ckpt) / "optim.pt", map_location="cpu", weights_only=False)
print(json.dumps({
    "logits": logits.float().tolist(),
    "trainer_keys": sorted(trainer),
    "optim_keys": sorted(optim),
    "n_optim_state": len(optim["state"]),
    "param_groups": [{k: (v if not isinstance(v, (list, tuple)) or k != "params" else len(v)) for k, v in g.items() if k in ("lr", "weight_decay", "params", "param_names")} for g in optim["param_groups"]],
}))
