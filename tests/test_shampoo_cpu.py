"""dense_optimizer='shampoo' wiring (the optional distributed_shampoo package is
not installed here): a stand-in package records the arguments the engine
passes and steps like SGD, so the engine's use of the optimizer is exercised."""
import os
import sys
import types

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class _Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def _install_fake(monkeypatch, with_momentum: bool):
    seen = {}

    class DistributedShampoo(torch.optim.SGD):
        if with_momentum:
            def __init__(self, params, lr=1e-3, betas=(0.9, 1.0), epsilon=1e-12, weight_decay=0.0,
                         max_preconditioner_dim=1024, precondition_frequency=1, start_preconditioning_step=1,
                         grafting_config=None, preconditioner_config=None, distributed_config=None,
                         momentum=0.0, use_nesterov=False, use_bias_correction=True,
                         use_decoupled_weight_decay=True):
                seen.update(dict(locals()))
                super().__init__(params, lr=lr)
        else:
            def __init__(self, params, lr=1e-3, betas=(0.9, 1.0), epsilon=1e-12, weight_decay=0.0,
                         max_preconditioner_dim=1024, precondition_frequency=1, start_preconditioning_step=1,
                         grafting_config=None, preconditioner_config=None, distributed_config=None):
                seen.update(dict(locals()))
                super().__init__(params, lr=lr)

    pkg = types.ModuleType("distributed_shampoo")
    pkg.DistributedShampoo = DistributedShampoo
    st = types.ModuleType("distributed_shampoo.shampoo_types")
    st.AdaGradPreconditionerConfig = _Cfg
    st.DDPDistributedConfig = _Cfg
    st.RootInvShampooPreconditionerConfig = _Cfg
    pre = types.ModuleType("distributed_shampoo.preconditioner")
    mf = types.ModuleType("distributed_shampoo.preconditioner.matrix_functions_types")
    mf.EigenConfig = _Cfg
    for name, mod in [("distributed_shampoo", pkg), ("distributed_shampoo.shampoo_types", st),
                      ("distributed_shampoo.preconditioner", pre),
                      ("distributed_shampoo.preconditioner.matrix_functions_types", mf)]:
        monkeypatch.setitem(sys.modules, name, mod)
    return seen


@pytest.mark.parametrize("with_momentum", [True, False])
def test_shampoo_engine_steps_with_reference_settings(monkeypatch, with_momentum):
    seen = _install_fake(monkeypatch, with_momentum)
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.training.engine import TrainEngine
    cfg = Config.load(os.path.join(ROOT, "configs", "onetrans_tiny.yaml"))
    cfg.train.dense_optimizer = "shampoo"
    cfg.train.kernels = "eager"
    cfg.train.bf16 = False
    tc = cfg.train
    tc.shampoo_use_bf16_factor_matrix = True
    tc.shampoo_use_ddp_distributed_config = True
    tc.shampoo_momentum = 0.5
    torch.manual_seed(0)
    model = build_model(cfg)
    eng = TrainEngine(model, cfg, torch.device("cpu"))
    before = [p.detach().clone() for p in eng.flat.params]
    loss, _ = eng.step(generate_batch(cfg, 16, seed=1))
    assert torch.isfinite(loss)
    assert any(not torch.equal(a, p.detach()) for a, p in zip(before, eng.flat.params))
    assert seen["lr"] == tc.lr and seen["betas"] == (0.9, 1.0) and seen["epsilon"] == 1e-4
    assert seen["precondition_frequency"] == seen["start_preconditioning_step"] == tc.shampoo_precondition_frequency
    assert seen["max_preconditioner_dim"] == tc.shampoo_max_preconditioner_dim
    assert seen["grafting_config"].epsilon == pytest.approx(1.4285714285714e-05)
    pc = seen["preconditioner_config"]
    assert pc.factor_matrix_dtype == torch.bfloat16 and pc.inverse_exponent_override == {1: 0.5, 2: 0.5}
    assert seen["distributed_config"].num_trainers_per_group == tc.shampoo_ddp_num_trainers_per_group
    if with_momentum:
        assert seen["momentum"] == 0.5 and seen["use_bias_correction"] is True
        assert seen["use_decoupled_weight_decay"] == tc.shampoo_use_decoupled_weight_decay


def test_shampoo_missing_package_is_a_clear_error(monkeypatch):
    monkeypatch.setitem(sys.modules, "distributed_shampoo", None)
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.training.engine import TrainEngine
    cfg = Config.load(os.path.join(ROOT, "configs", "onetrans_tiny.yaml"))
    cfg.train.dense_optimizer = "shampoo"
    with pytest.raises(RuntimeError, match="distributed_shampoo"):
        TrainEngine(build_model(cfg), cfg, torch.device("cpu"))
