"""qwenquest_b200 — B200-native (sm_100a) Quest sparse-decode path for QwenQuest.

Drop-in attention backends for the reference's ``Engine``:

* :class:`~qwenquest_b200.backends.B200QuestOnlyBackend` (``attention_mode="quest"``)
* :class:`~qwenquest_b200.backends.B200QuestHiSparseBackend` (``attention_mode="quest_hisparse"``)

plus :class:`~qwenquest_b200.quest.QuestAlgorithm` and
:class:`~qwenquest_b200.hisparse.HiSparseCoordinator` with the reference's
APIs, and :class:`~qwenquest_b200.graphs.DecodeStepGraph` (a decode step
captured in a CUDA graph); :class:`~qwenquest_b200.moe.B200SparseMoeBlock` and
:func:`~qwenquest_b200.moe.install_moe` (the model's MoE blocks on the tensor
cores).  All decode work runs in hand-written CUDA kernels in ``libqquest.so``
(C ABI: ``include/qquest.h``); nothing falls back to the CPU.  Importing this
package does not load the library; the first backend / algorithm object does.
"""

__version__ = "0.1.0"

__all__ = [
    "B200QuestHiSparseBackend",
    "B200QuestOnlyBackend",
    "B200SparseMoeBlock",
    "DecodeStepGraph",
    "HiSparseCoordinator",
    "QuestAlgorithm",
    "QuestTrace",
    "install_moe",
]


def __getattr__(name):
    if name in ("B200QuestHiSparseBackend", "B200QuestOnlyBackend"):
        from qwenquest_b200 import backends

        return getattr(backends, name)
    if name in ("B200SparseMoeBlock", "install_moe"):
        from qwenquest_b200 import moe

        return getattr(moe, name)
    if name == "DecodeStepGraph":
        from qwenquest_b200.graphs import DecodeStepGraph

        return DecodeStepGraph
    if name == "HiSparseCoordinator":
        from qwenquest_b200.hisparse import HiSparseCoordinator

        return HiSparseCoordinator
    if name in ("QuestAlgorithm", "QuestTrace"):
        from qwenquest_b200 import quest

        return getattr(quest, name)
    raise AttributeError(name)
