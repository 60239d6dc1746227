// graph_loop.cu -- device-side decode loops inside one CUDA graph.
//
// The reference drives decoding from Python: every STD round ends with host
// reads of the verify argmax and of the accepted length (std_qwen25vl.py:806
// `.tolist()`, the `while len(generated) < max_new_tokens` loop at :766), so the
// GPU idles while the host decides whether to run another round.  Here the loop
// itself lives in the graph: a WHILE conditional node whose body is one decode
// round (or one AR step) and whose condition a one-warp kernel sets from the
// device-resident `done` flags at the end of every iteration.  The host
// launches the whole decode once and synchronises once.
//
// Capture protocol (the stream is already capturing, e.g. under
// torch.cuda.graph):
//   std_capture_while_begin(stream, body_stream, done, B, counter)
//     enqueues loop_init_kernel on `stream` (counter = 0; condition = "some
//     request is still running"), appends the WHILE node after it, and starts
//     capturing `body_stream` into the node's body graph;
//   ... the caller enqueues one round on body_stream ...
//   std_capture_while_end(body_stream, done, B, counter, max_iters)
//     enqueues loop_continue_kernel on body_stream (counter += 1; condition =
//     "some request running and counter < max_iters") and ends the body
//     capture.
// The iteration bound makes every loop finite whatever the done flags say.
#include "common.cuh"

namespace stdb {

// 1 when some request b < B has done[b] == 0.
STD_DEV unsigned any_running(const int32_t* done, int B) {
  unsigned run = 0;
  for (int b = threadIdx.x; b < B; b += 32) run |= (done[b] == 0) ? 1u : 0u;
  return __any_sync(0xffffffffu, run != 0) ? 1u : 0u;
}

__global__ void loop_init_kernel(cudaGraphConditionalHandle h, const int32_t* done, int B, int32_t* counter) {
  const unsigned run = any_running(done, B);
  if (threadIdx.x == 0) {
    *counter = 0;
    cudaGraphSetConditional(h, run);
  }
}

__global__ void loop_continue_kernel(cudaGraphConditionalHandle h, const int32_t* done, int B, int32_t* counter,
                                     int max_iters) {
  const unsigned run = any_running(done, B);
  if (threadIdx.x == 0) {
    const int32_t c = *counter + 1;
    *counter = c;
    cudaGraphSetConditional(h, (run != 0u && c < max_iters) ? 1u : 0u);
  }
}

}  // namespace stdb

extern "C" int std_capture_while_begin(void* stream, void* body_stream, const int32_t* done, int B, int32_t* counter,
                                       unsigned long long* handle_out, void** body_graph_out) {
  if (stream == nullptr || body_stream == nullptr || stream == body_stream || done == nullptr || counter == nullptr ||
      B <= 0 || handle_out == nullptr)
    return 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaGraph_t graph = nullptr;
  if (cudaStreamGetCaptureInfo(s, &st, nullptr, &graph, nullptr, nullptr) != cudaSuccess) return 4;
  if (st != cudaStreamCaptureStatusActive || graph == nullptr) return 1;  // must be called while capturing
  cudaGraphConditionalHandle h;
  // default 0: if the init kernel never ran, the body does not run either
  if (cudaGraphConditionalHandleCreate(&h, graph, 0, cudaGraphCondAssignDefault) != cudaSuccess) return 4;
  count_launch();
  stdb::loop_init_kernel<<<1, 32, 0, s>>>(h, done, B, counter);
  if (cudaGetLastError() != cudaSuccess) return 4;
  const cudaGraphNode_t* deps = nullptr;
  size_t ndeps = 0;
  if (cudaStreamGetCaptureInfo(s, &st, nullptr, &graph, &deps, &ndeps) != cudaSuccess) return 4;
  cudaGraphNodeParams np = {};
  np.type = cudaGraphNodeTypeConditional;
  np.conditional.handle = h;
  np.conditional.type = cudaGraphCondTypeWhile;
  np.conditional.size = 1;
  cudaGraphNode_t node;
  if (cudaGraphAddNode(&node, graph, deps, ndeps, &np) != cudaSuccess) return 4;
  if (cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies) != cudaSuccess) return 4;
  cudaGraph_t body = np.conditional.phGraph_out[0];
  if (cudaStreamBeginCaptureToGraph(static_cast<cudaStream_t>(body_stream), body, nullptr, nullptr, 0,
                                    cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return 4;
  *handle_out = static_cast<unsigned long long>(h);
  if (body_graph_out != nullptr) *body_graph_out = body;
  return 0;
}

extern "C" int std_capture_while_end(void* body_stream, unsigned long long handle, const int32_t* done, int B,
                                     int32_t* counter, int max_iters) {
  if (body_stream == nullptr || done == nullptr || counter == nullptr || B <= 0 || max_iters <= 0) return 1;
  cudaStream_t s = static_cast<cudaStream_t>(body_stream);
  count_launch();
  stdb::loop_continue_kernel<<<1, 32, 0, s>>>(static_cast<cudaGraphConditionalHandle>(handle), done, B, counter,
                                               max_iters);
  const cudaError_t launch = cudaGetLastError();
  cudaGraph_t g = nullptr;
  const cudaError_t end = cudaStreamEndCapture(s, &g);  // the body graph is owned by the WHILE node
  return (launch == cudaSuccess && end == cudaSuccess) ? 0 : 4;
}

// IF node: a conditional handle in the graph `stream` is capturing (for a
// kernel that sets it), then the node after the stream's current work, with
// `body_stream` capturing its body until std_capture_if_end.
extern "C" int std_graph_cond_handle(void* stream, unsigned long long* handle_out) {
  if (stream == nullptr || handle_out == nullptr) return 1;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaGraph_t graph = nullptr;
  if (cudaStreamGetCaptureInfo(static_cast<cudaStream_t>(stream), &st, nullptr, &graph, nullptr, nullptr) !=
      cudaSuccess)
    return 4;
  if (st != cudaStreamCaptureStatusActive || graph == nullptr) return 1;
  cudaGraphConditionalHandle h;
  if (cudaGraphConditionalHandleCreate(&h, graph, 0, cudaGraphCondAssignDefault) != cudaSuccess) return 4;
  *handle_out = static_cast<unsigned long long>(h);
  return 0;
}

extern "C" int std_capture_if_begin(void* stream, void* body_stream, unsigned long long handle) {
  if (stream == nullptr || body_stream == nullptr || stream == body_stream) return 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  size_t ndeps = 0;
  if (cudaStreamGetCaptureInfo(s, &st, nullptr, &graph, &deps, &ndeps) != cudaSuccess) return 4;
  if (st != cudaStreamCaptureStatusActive || graph == nullptr) return 1;
  cudaGraphNodeParams np = {};
  np.type = cudaGraphNodeTypeConditional;
  np.conditional.handle = static_cast<cudaGraphConditionalHandle>(handle);
  np.conditional.type = cudaGraphCondTypeIf;
  np.conditional.size = 1;
  cudaGraphNode_t node;
  if (cudaGraphAddNode(&node, graph, deps, ndeps, &np) != cudaSuccess) return 4;
  if (cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies) != cudaSuccess) return 4;
  if (cudaStreamBeginCaptureToGraph(static_cast<cudaStream_t>(body_stream), np.conditional.phGraph_out[0], nullptr,
                                    nullptr, 0, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return 4;
  return 0;
}

extern "C" int std_capture_if_end(void* body_stream) {
  if (body_stream == nullptr) return 1;
  cudaGraph_t g = nullptr;
  return cudaStreamEndCapture(static_cast<cudaStream_t>(body_stream), &g) == cudaSuccess ? 0 : 4;
}

// A stream of its own for capturing a conditional body (non-blocking, never
// destroyed): torch hands out pooled streams, so two of its streams can be
// the same CUDA stream, and a body must be captured on a stream that is not
// the one capturing its parent graph.
extern "C" int std_stream_create(void** stream_out) {
  if (stream_out == nullptr) return 1;
  cudaStream_t s = nullptr;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return 4;
  *stream_out = s;
  return 0;
}

extern "C" long long std_launch_count(void) { return g_std_launches.load(std::memory_order_relaxed); }
