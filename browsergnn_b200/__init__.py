"""browsergnn_b200: a B200 (sm_100a) backend for BrowserGNN's message-passing path.

The compute lives in libbgnn_cuda.so (include/bgnn.h); this package is the
host-side mirror of the reference's API for that path:

  GraphData, batchGraphs, fromEdgeList          src/core/graph.ts
  SparseCOO, SparseCSR, MessagePassing,
  computeGCNNorm                                src/core/sparse.ts
  GPUSparse, GPUTensor, isGPUAvailable          src/core/gpu-sparse.ts
  initBrowserGNN, getBackend, getComputeManager src/backend/index.ts
  CudaComputeManager                            (WebGPUComputeManager's method set)
  GCNConv, GATConv, SAGEConv, GINConv           src/layers/*.ts
  Linear, ReLU, ELU, LeakyReLU, Sigmoid, Tanh,
  GELU, SiLU, PReLU, Softmax, LogSoftmax,
  Dropout, Sequential, Module                   src/nn/*.ts
  StudentMasteryPredictor,
  LearningPathRecommender,
  ConceptPrerequisiteMapper                     src/models/*.ts
  serializeModel, loadModelFromJSON, ...        src/utils/serialization.ts
"""
from ._lib import BGNNError, BGNNIndexError
from .backend import (CudaComputeManager, get_backend, get_compute_manager, get_context,
                      getBackend, getComputeManager, init_browsergnn, initBrowserGNN,
                      is_gpu_available, isGPUAvailable, to_host)
from .graph import DeviceGraph, GraphData, batch_graphs, batchGraphs, from_edge_list, fromEdgeList
from .layers import (ELU, GATConv, GCNConv, GINConv, LeakyReLU, Module, ReLU, SAGEConv,
                     Sequential, global_sum_pool)
from .ops import (GPUSparse, GPUTensor, MessagePassing, SparseCOO, SparseCSR, compute_gcn_norm,
                  computeGCNNorm)
from .nn import (GELU, Dropout, Linear, LogSoftmax, PReLU, SiLU, Sigmoid, Softmax, Tanh,
                 manual_seed)
from .models import ConceptPrerequisiteMapper, LearningPathRecommender, StudentMasteryPredictor
from . import serialization
from .graphs import CapturedForward
from .serialization import (deserializeModel, getModelSize, getStateDict, loadModelFromJSON,
                            loadStateDict, saveModelToJSON, serializeModel)

__all__ = [
    "BGNNError", "BGNNIndexError", "CudaComputeManager", "DeviceGraph", "ELU", "GATConv",
    "GCNConv", "GINConv", "GPUSparse", "GPUTensor", "GraphData", "LeakyReLU", "MessagePassing",
    "Module", "ReLU", "SAGEConv", "Sequential", "SparseCOO", "SparseCSR", "batchGraphs",
    "batch_graphs", "computeGCNNorm", "compute_gcn_norm", "fromEdgeList", "from_edge_list",
    "getBackend", "getComputeManager", "get_backend", "get_compute_manager", "get_context",
    "to_host",
    "global_sum_pool", "initBrowserGNN", "init_browsergnn", "isGPUAvailable", "is_gpu_available",
    "Linear", "Sigmoid", "Tanh", "GELU", "SiLU", "PReLU", "Softmax", "LogSoftmax", "Dropout",
    "manual_seed", "StudentMasteryPredictor", "LearningPathRecommender",
    "ConceptPrerequisiteMapper", "serialization", "serializeModel", "deserializeModel",
    "saveModelToJSON", "loadModelFromJSON", "getStateDict", "loadStateDict", "getModelSize",
    "CapturedForward",
]
