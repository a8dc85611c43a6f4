// Request batcher: the batch-capable serving surface over one engine.
//
// The reference serialises every predict of a model on Runtime::mutex
// (src/models/gwp05/model.cpp:61) and advertises no batch capability
// (Capabilities::batch_inference, include/wam/types.h:236-237), so concurrent
// sessions queue one chunk at a time. Here any number of client threads call
// wam_b200_batcher_predict concurrently; one worker thread per engine takes
// the queued requests in arrival order, up to the engine's max_batch, waiting
// at most max_wait_us after the first for more to arrive, and runs them as one
// wam_b200_predict_batch (one prefix + one denoise program over the batch).
// If a batch fails, its requests are retried one by one so that a bad request
// fails alone. Each caller gets its own chunk, status and the size of the
// batch it rode in.
#include <cuda_runtime.h>

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "c_api_util.h"
#include "wam_b200.h"

namespace {

struct Item {
  const wam_b200_request* req = nullptr;
  float* out = nullptr;
  size_t out_n = 0;
  int rc = 0;
  std::string msg;
  wam_b200_stats stats{};
  int batch = 0;
  bool done = false;
};

int bfail(wam_b200_status* st, int code, const std::string& msg) {
  wamb::set_last_error(msg);
  if (st) {
    st->code = code;
    st->message = static_cast<char*>(std::malloc(msg.size() + 1));
    if (st->message) std::memcpy(st->message, msg.c_str(), msg.size() + 1);
  }
  return code;
}

}  // namespace

struct wam_b200_batcher {
  wam_b200_engine* engine = nullptr;
  int max_batch = 1;
  int max_wait_us = 0;
  size_t chunk = 0;  // floats of one action chunk
  std::mutex m;
  std::condition_variable cv_work, cv_done;
  std::deque<Item*> queue;
  bool stop = false;
  long long batches = 0, requests = 0;
  std::thread worker;

  void run_batch(std::vector<Item*>& items) {
    const int n = static_cast<int>(items.size());
    std::vector<wam_b200_request> reqs(n);
    for (int i = 0; i < n; ++i) reqs[i] = *items[i]->req;
    std::vector<float> out(static_cast<size_t>(n) * chunk);
    wam_b200_stats s{};
    wam_b200_status st{0, nullptr};
    int rc = wam_b200_predict_batch(engine, reqs.data(), n, out.data(), out.size(), &s, &st);
    if (rc == WAM_B200_OK) {
      for (int i = 0; i < n; ++i) {
        std::memcpy(items[i]->out, out.data() + static_cast<size_t>(i) * chunk, chunk * sizeof(float));
        items[i]->rc = WAM_B200_OK;
        items[i]->stats = s;
        items[i]->batch = n;
      }
      wam_b200_status_free(&st);
      return;
    }
    wam_b200_status_free(&st);
    // Isolate the failing request(s): one by one.
    for (int i = 0; i < n; ++i) {
      wam_b200_status s1{0, nullptr};
      wam_b200_stats one{};
      const int r1 = wam_b200_predict(engine, &reqs[i], items[i]->out, chunk, &one, &s1);
      items[i]->rc = r1;
      items[i]->msg = s1.message ? s1.message : "";
      items[i]->stats = one;
      items[i]->batch = 1;
      wam_b200_status_free(&s1);
    }
  }

  void loop() {
    std::unique_lock<std::mutex> lk(m);
    while (true) {
      cv_work.wait(lk, [&] { return stop || !queue.empty(); });
      if (queue.empty()) {
        if (stop) return;
        continue;
      }
      if (max_wait_us > 0 && static_cast<int>(queue.size()) < max_batch && !stop) {
        const auto until = std::chrono::steady_clock::now() + std::chrono::microseconds(max_wait_us);
        cv_work.wait_until(lk, until,
                           [&] { return stop || static_cast<int>(queue.size()) >= max_batch; });
      }
      std::vector<Item*> items;
      while (!queue.empty() && static_cast<int>(items.size()) < max_batch) {
        items.push_back(queue.front());
        queue.pop_front();
      }
      lk.unlock();
      run_batch(items);
      lk.lock();
      ++batches;
      requests += static_cast<long long>(items.size());
      for (Item* it : items) it->done = true;
      cv_done.notify_all();
    }
  }
};

extern "C" {

WAM_B200_API int wam_b200_batcher_create(wam_b200_engine* engine, int max_wait_us,
                                         wam_b200_batcher** out, wam_b200_status* st) {
  if (!engine || !out) return bfail(st, WAM_B200_INVALID_ARGUMENT, "engine and batcher pointer are required");
  if (max_wait_us < 0 || max_wait_us > 10000000)
    return bfail(st, WAM_B200_INVALID_ARGUMENT, "max_wait_us must be in [0, 10 s]");
  wam_b200_geometry g{};
  if (wam_b200_geometry_of(engine, &g) != WAM_B200_OK)
    return bfail(st, WAM_B200_INVALID_ARGUMENT, "engine geometry unavailable");
  auto* b = new wam_b200_batcher();
  b->engine = engine;
  b->max_batch = wam_b200_max_batch(engine);
  b->max_wait_us = max_wait_us;
  b->chunk = static_cast<size_t>(g.action_chunk) * g.real_action_dim;
  b->worker = std::thread([b] { b->loop(); });
  *out = b;
  if (st) {
    st->code = WAM_B200_OK;
    st->message = nullptr;
  }
  return WAM_B200_OK;
}

WAM_B200_API void wam_b200_batcher_destroy(wam_b200_batcher* b) {
  if (!b) return;
  {
    std::lock_guard<std::mutex> lk(b->m);
    b->stop = true;
  }
  b->cv_work.notify_all();
  if (b->worker.joinable()) b->worker.join();
  delete b;
}

WAM_B200_API int wam_b200_batcher_predict(wam_b200_batcher* b, const wam_b200_request* request,
                                          float* action_out, size_t action_out_n,
                                          wam_b200_stats* stats, int* batch_size,
                                          wam_b200_status* st) {
  if (!b || !request || !action_out)
    return bfail(st, WAM_B200_INVALID_ARGUMENT, "batcher, request and output are required");
  if (action_out_n < b->chunk) return bfail(st, WAM_B200_INVALID_ARGUMENT, "action output buffer is too small");
  Item it;
  it.req = request;
  it.out = action_out;
  it.out_n = action_out_n;
  {
    std::unique_lock<std::mutex> lk(b->m);
    if (b->stop) return bfail(st, WAM_B200_INVALID_ARGUMENT, "batcher is shutting down");
    b->queue.push_back(&it);
    b->cv_work.notify_one();
    b->cv_done.wait(lk, [&] { return it.done; });
  }
  if (stats) *stats = it.stats;
  if (batch_size) *batch_size = it.batch;
  if (it.rc != WAM_B200_OK) return bfail(st, it.rc, it.msg.empty() ? "predict failed" : it.msg);
  if (st) {
    st->code = WAM_B200_OK;
    st->message = nullptr;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_batcher_counts(wam_b200_batcher* b, long long* batches,
                                         long long* requests) {
  if (!b) return WAM_B200_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(b->m);
  if (batches) *batches = b->batches;
  if (requests) *requests = b->requests;
  return WAM_B200_OK;
}

}  // extern "C"
