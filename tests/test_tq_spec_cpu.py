"""Data-plane sizing (CPU): the column store's partition holds every sample in flight -- batches the trainer
has not consumed plus rollouts still generating -- ``max(4 * batch, 2 * max_running + batch, 1024)``, and the
environment override wins."""

from meshy_b200.config import InferenceServiceConfig, RolloutServiceConfig, TrainerConfig, TrainingServiceConfig
from meshy_b200.service.base import ServiceGroup
from meshy_b200.tq.launch import derive_spec


def _groups(batch, max_running):
    return [ServiceGroup(id="actor_infer", n_replicas=1, n_gpus_per_replica=1,
                         config=InferenceServiceConfig(model_path="m")),
            ServiceGroup(id="actor_train", n_replicas=1, n_gpus_per_replica=1,
                         config=TrainingServiceConfig(model_path="m", trainer_config=TrainerConfig(),
                                                      batch_size=batch)),
            ServiceGroup(id="rollout", n_replicas=1, n_gpus_per_replica=0,
                         config=RolloutServiceConfig(model_path="m", dataset="d:D",
                                                     async_max_running_request=max_running))]


def test_sizing(tmp_path, monkeypatch):
    monkeypatch.delenv("XRL_TQ_PRE_ALLOC", raising=False)
    assert derive_spec(_groups(2048, -1), str(tmp_path))["pre_alloc_sample_num"] == 4 * 2048
    assert derive_spec(_groups(64, 3072), str(tmp_path))["pre_alloc_sample_num"] == 2 * 3072 + 64
    assert derive_spec(_groups(4, -1), str(tmp_path))["pre_alloc_sample_num"] == 1024
    monkeypatch.setenv("XRL_TQ_PRE_ALLOC", "77")
    assert derive_spec(_groups(2048, -1), str(tmp_path))["pre_alloc_sample_num"] == 77
