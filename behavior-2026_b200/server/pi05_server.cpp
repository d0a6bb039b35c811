// pi05_server.cpp — policy server over the engine's C ABI (the reference's server/pi05_server.cpp,
// docs/archive/windows/π05_네이티브엔진.md:120-123 and :314-329): openpi's WebSocket protocol, one engine
// per process, one pi05_act_batch call per request for all the environments the request carries.
//
// Protocol (openpi serving/websocket_policy_server.py as the evaluator's WebsocketClientPolicy speaks it):
//   * GET /healthz answers 200 "OK"; any other request must be a WebSocket upgrade (RFC 6455);
//   * on connect the server sends its metadata (a msgpack map);
//   * each binary message is a msgpack observation map whose arrays use openpi's msgpack_numpy form;
//     the reply is {"action": f32 array, "server_timing": {"infer_ms": ..}};
//   * {"reset": true} (optionally with "env_ids") forgets the environments' chunks (pi05_reset_slot);
//   * "__action_chunk_size__": K returns the next K actions of each environment's receding-horizon plan
//     at once ([K][act_dim] per environment), warning when K exceeds the re-plan period (the K steps
//     then span two plans, all made from this observation).
// Observation keys: one uint8 image per camera key ([H][W][3 or 4] at any size, or [n][H][W][C] for n
// environments), "tokens" int32 [n_text] or [n][n_text] (token ids: the tokenizer's model file is not part
// of this build), optional "state" f32 [act_dim] / [n][act_dim], "noise" f32 [horizon][32] / [n][..],
// "env_ids" int [n] (slots; default 0..n-1).
// Sockets use TCP_NODELAY and re-arm TCP_QUICKACK after every read, as the reference did.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <sstream>
#include <thread>

#include "../../include/pi05.h"
#include "wire.h"

namespace {

struct Options {
  int port = 8000;
  std::string host = "0.0.0.0";
  std::string weights;
  long random_seed = -1;
  int device = 0, max_batch = 8;
  pi05_config cfg;
  int act_dim = 23, replan = 16;
  std::vector<float> mean, stdv;
  std::vector<uint8_t> delta;
  uint64_t noise_seed = 0;
  std::vector<std::string> cameras = {"head", "left_wrist", "right_wrist"};
};

std::mutex g_engine_mu;  // calls on one engine are not re-entrant

template <typename T>
std::vector<T> parse_list(const std::string& s) {
  std::vector<T> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ',')) out.push_back((T)std::stod(item));
  return out;
}

std::vector<std::string> split(const std::string& s) {
  std::vector<std::string> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ',')) out.push_back(item);
  return out;
}

// ---------------------------------------------------------------- socket I/O
bool read_exact(int fd, void* buf, size_t n) {
  char* p = (char*)buf;
  while (n) {
    const ssize_t r = recv(fd, p, n, 0);
    if (r <= 0) return false;
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_QUICKACK, &one, sizeof one);
    p += r;
    n -= (size_t)r;
  }
  return true;
}

bool write_all(int fd, const std::string& s) {
  size_t at = 0;
  while (at < s.size()) {
    const ssize_t w = send(fd, s.data() + at, s.size() - at, MSG_NOSIGNAL);
    if (w <= 0) return false;
    at += (size_t)w;
  }
  return true;
}

// One whole message (continuation frames joined); answers pings; false on close or error.
bool ws_read_message(int fd, std::string& msg, int& opcode) {
  msg.clear();
  opcode = -1;
  for (;;) {
    uint8_t h[2];
    if (!read_exact(fd, h, 2)) return false;
    const bool fin = h[0] & 0x80;
    const int op = h[0] & 0x0f;
    const bool masked = h[1] & 0x80;
    uint64_t n = h[1] & 0x7f;
    if (n == 126) {
      uint8_t e[2];
      if (!read_exact(fd, e, 2)) return false;
      n = (uint64_t)e[0] << 8 | e[1];
    } else if (n == 127) {
      uint8_t e[8];
      if (!read_exact(fd, e, 8)) return false;
      n = 0;
      for (int i = 0; i < 8; ++i) n = n << 8 | e[i];
    }
    if (!masked || n > (1ull << 31)) return false;  // clients mask every frame (RFC 6455 5.1)
    uint8_t key[4];
    if (!read_exact(fd, key, 4)) return false;
    std::string payload(n, '\0');
    if (n && !read_exact(fd, &payload[0], n)) return false;
    for (uint64_t i = 0; i < n; ++i) payload[i] ^= (char)key[i & 3];
    if (op == 0x8) {
      write_all(fd, wire::ws_frame(0x8, ""));
      return false;
    }
    if (op == 0x9) {
      if (!write_all(fd, wire::ws_frame(0xA, payload))) return false;
      continue;
    }
    if (op == 0xA) continue;
    if (op != 0) opcode = op;
    msg += payload;
    if (fin) return true;
  }
}

bool send_value(int fd, const wire::VPtr& v) {
  std::string out;
  wire::pack(out, *v);
  return write_all(fd, wire::ws_frame(0x2, out));
}

// ---------------------------------------------------------------- requests
std::string error_text(pi05_engine* e, int rc) {
  return std::string("pi05 error ") + std::to_string(rc) + ": " + pi05_last_error(e);
}

wire::VPtr error_reply(const std::string& why) {
  auto m = wire::v_map();
  wire::put(m, "error", wire::v_str(why));
  return m;
}

// An array whose byte count matches its dtype and shape.
bool array_of(const wire::Value* v, const char* dtype, size_t itemsize, wire::NdArray* a) {
  return wire::as_ndarray(v, a) && a->dtype == dtype && a->data.size() == (size_t)a->size() * itemsize;
}

// Leading environment count n of an array whose per-environment rank is `rank` (n = 1 without it).
bool env_count(const wire::NdArray& a, size_t rank, int64_t* n) {
  if (a.shape.size() == rank) {
    *n = 1;
    return true;
  }
  if (a.shape.size() == rank + 1) {
    *n = a.shape[0];
    return true;
  }
  return false;
}

wire::VPtr handle_obs(pi05_engine* e, const Options& o, const wire::Value& obs) {
  const int ncam = (int)o.cameras.size();
  std::vector<wire::NdArray> cams(ncam);
  int64_t n = -1;
  for (int c = 0; c < ncam; ++c) {
    if (!array_of(obs.get(o.cameras[c]), "|u1", 1, &cams[c]))
      return error_reply("observation lacks uint8 camera image '" + o.cameras[c] + "'");
    int64_t k;
    if (!env_count(cams[c], 3, &k) || (n >= 0 && k != n)) return error_reply("camera images disagree in shape");
    n = k;
  }
  if (n < 1 || n > o.max_batch) return error_reply("1 .. max_batch environments per request");
  const bool batched = cams[0].shape.size() == 4;
  wire::NdArray tok, st, nz, ids;
  const bool has_tok = array_of(obs.get("tokens"), "<i4", 4, &tok);
  if (o.cfg.n_text > 0 && (!has_tok || tok.size() != n * o.cfg.n_text))
    return error_reply("observation lacks int32 'tokens' of n_text ids per environment");
  const bool has_state = obs.get("state") != nullptr;
  if (has_state && (!array_of(obs.get("state"), "<f4", 4, &st) || st.size() != n * o.act_dim))
    return error_reply("'state' must be float32 with act_dim values per environment");
  const bool has_noise = obs.get("noise") != nullptr;
  if (has_noise && (!array_of(obs.get("noise"), "<f4", 4, &nz) || nz.size() != n * o.cfg.horizon * 32))
    return error_reply("'noise' must be float32 [horizon][32] per environment");
  std::vector<int> slots(n);
  for (int i = 0; i < n; ++i) slots[i] = i;
  if (obs.get("env_ids")) {
    if (!(array_of(obs.get("env_ids"), "<i8", 8, &ids) || array_of(obs.get("env_ids"), "<i4", 4, &ids)) ||
        ids.size() != n)
      return error_reply("'env_ids' must be n ints");
    for (int i = 0; i < n; ++i)
      slots[i] = ids.dtype == "<i8" ? (int)((const int64_t*)ids.data.data())[i] : ((const int32_t*)ids.data.data())[i];
  }
  int K = 1;
  bool chunk = false;
  if (const wire::Value* k = obs.get("__action_chunk_size__")) {
    if (k->kind != wire::Value::INT || k->i < 1 || k->i > o.cfg.horizon) return error_reply("bad __action_chunk_size__");
    K = (int)k->i;
    chunk = true;
  }
  std::vector<pi05_frame> frames((size_t)n * ncam);
  for (int i = 0; i < n; ++i)
    for (int c = 0; c < ncam; ++c) {
      const wire::NdArray& a = cams[c];
      const size_t r = batched ? 1 : 0;
      pi05_frame& f = frames[(size_t)i * ncam + c];
      f.height = (int32_t)a.shape[r];
      f.width = (int32_t)a.shape[r + 1];
      f.channels = (int32_t)a.shape[r + 2];
      f.stride = (int64_t)f.width * f.channels;
      f.data = a.data.data() + (size_t)i * f.height * f.stride;
    }
  std::vector<float> out((size_t)n * K * o.act_dim), row((size_t)n * o.act_dim);
  const auto t0 = std::chrono::steady_clock::now();
  {
    std::lock_guard<std::mutex> lk(g_engine_mu);
    for (int k = 0; k < K; ++k) {
      const int rc = pi05_act_batch(e, (int)n, slots.data(), frames.data(),
                                    has_tok ? (const int32_t*)tok.data.data() : nullptr,
                                    has_state ? (const float*)st.data.data() : nullptr,
                                    has_noise ? (const float*)nz.data.data() : nullptr, row.data());
      if (rc != PI05_OK) return error_reply(error_text(e, rc));
      for (int i = 0; i < n; ++i)
        memcpy(&out[((size_t)i * K + k) * o.act_dim], &row[(size_t)i * o.act_dim], o.act_dim * sizeof(float));
    }
  }
  const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (chunk && K > o.replan) fprintf(stderr, "pi05_server: an action chunk of %d steps spans a re-plan\n", K);
  std::vector<int64_t> shape;
  if (batched) shape.push_back(n);
  if (chunk) shape.push_back(K);
  shape.push_back(o.act_dim);
  auto reply = wire::v_map();
  wire::put(reply, "action", wire::v_ndarray("<f4", shape, out.data(), out.size() * sizeof(float)));
  auto timing = wire::v_map();
  wire::put(timing, "infer_ms", wire::v_float(ms));
  wire::put(reply, "server_timing", timing);
  return reply;
}

wire::VPtr metadata(pi05_engine* e, const Options& o) {
  auto m = wire::v_map();
  wire::put(m, "kind", wire::v_str("pi05"));
  wire::put(m, "horizon", wire::v_int(o.cfg.horizon));
  wire::put(m, "act_dim", wire::v_int(o.act_dim));
  wire::put(m, "replan", wire::v_int(o.replan));
  wire::put(m, "n_text", wire::v_int(o.cfg.n_text));
  wire::put(m, "max_batch", wire::v_int(o.max_batch));
  wire::put(m, "prefix_len", wire::v_int(pi05_prefix_len(e)));
  auto cams = wire::v_array();
  for (const std::string& c : o.cameras) cams->arr.push_back(wire::v_str(c));
  wire::put(m, "camera_keys", cams);
  return m;
}

void serve(int fd, pi05_engine* e, const Options& o) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
  std::string req;
  char c;
  while (req.size() < 65536 && req.find("\r\n\r\n") == std::string::npos) {
    if (!read_exact(fd, &c, 1)) return;
    req.push_back(c);
  }
  if (req.rfind("GET /healthz", 0) == 0) {
    write_all(fd, "HTTP/1.1 200 OK\r\nContent-Type: text/plain\r\nContent-Length: 3\r\nConnection: close\r\n\r\nOK\n");
    return;
  }
  std::string key;
  std::istringstream hs(req);
  std::string line;
  while (std::getline(hs, line)) {
    if (!line.empty() && line.back() == '\r') line.pop_back();
    const size_t colon = line.find(':');
    if (colon == std::string::npos) continue;
    std::string name = line.substr(0, colon);
    for (char& ch : name) ch = (char)tolower(ch);
    if (name == "sec-websocket-key") {
      key = line.substr(colon + 1);
      key.erase(0, key.find_first_not_of(" \t"));
      key.erase(key.find_last_not_of(" \t") + 1);
    }
  }
  if (key.empty()) {
    write_all(fd, "HTTP/1.1 400 Bad Request\r\nContent-Length: 0\r\nConnection: close\r\n\r\n");
    return;
  }
  if (!write_all(fd, "HTTP/1.1 101 Switching Protocols\r\nUpgrade: websocket\r\nConnection: Upgrade\r\n"
                     "Sec-WebSocket-Accept: " + wire::ws_accept(key) + "\r\n\r\n"))
    return;
  if (!send_value(fd, metadata(e, o))) return;
  std::string msg;
  int op;
  while (ws_read_message(fd, msg, op)) {
    wire::VPtr reply;
    try {
      wire::Reader rd((const uint8_t*)msg.data(), msg.size());
      wire::VPtr obs = rd.value();
      if (obs->kind != wire::Value::MAP) {
        reply = error_reply("expected a msgpack map");
      } else if (const wire::Value* r = obs->get("reset"); r && r->kind == wire::Value::BOOL && r->b) {
        wire::NdArray ids;
        std::lock_guard<std::mutex> lk(g_engine_mu);
        if (array_of(obs->get("env_ids"), "<i8", 8, &ids)) {
          for (int64_t i = 0; i < ids.size(); ++i) pi05_reset_slot(e, (int)((const int64_t*)ids.data.data())[i]);
        } else {
          for (int s = 0; s < o.max_batch; ++s) pi05_reset_slot(e, s);
        }
        reply = wire::v_map();
        wire::put(reply, "reset", wire::v_bool(true));
      } else {
        reply = handle_obs(e, o, *obs);
      }
    } catch (const std::exception& ex) {
      reply = error_reply(ex.what());
    }
    if (!send_value(fd, reply)) return;
  }
}

// ---------------------------------------------------------------- self-test of the wire formats
int selftest() {
  int bad = 0;
  auto hex = [](const std::string& s) {
    static const char* d = "0123456789abcdef";
    std::string o;
    for (unsigned char c : s) o += d[c >> 4], o += d[c & 15];
    return o;
  };
  bad += hex(wire::sha1("abc")) != "a9993e364706816aba3e25717850c26c9cd0d89d";
  bad += hex(wire::sha1("")) != "da39a3ee5e6b4b0d3255bfef95601890afd80709";
  bad += wire::base64("foobar") != "Zm9vYmFy" || wire::base64("fooba") != "Zm9vYmE=" || wire::base64("foob") != "Zm9vYg==";
  bad += wire::ws_accept("dGhlIHNhbXBsZSBub25jZQ==") != "s3pPLMBiTxaQ9kYGzzhZRbK+xOo=";  // RFC 6455 section 1.3
  auto m = wire::v_map();
  const float xs[3] = {1.5f, -2.0f, 3.25f};
  wire::put(m, "a", wire::v_ndarray("<f4", {3}, xs, sizeof xs));
  wire::put(m, "k", wire::v_int(-70000));
  wire::put(m, "s", wire::v_str(std::string(40, 'x')));
  std::string buf;
  wire::pack(buf, *m);
  wire::Reader rd((const uint8_t*)buf.data(), buf.size());
  wire::VPtr back = rd.value();
  wire::NdArray a;
  bad += !wire::as_ndarray(back->get("a"), &a) || a.size() != 3 || memcmp(a.data.data(), xs, sizeof xs) != 0;
  bad += back->get("k")->i != -70000 || back->get("s")->s != std::string(40, 'x') || rd.used() != buf.size();
  printf(bad ? "selftest FAILED (%d)\n" : "selftest ok\n", bad);
  return bad ? 1 : 0;
}

void usage() {
  fprintf(stderr,
          "pi05_server [--weights FILE | --random-weights SEED] [--port 8000] [--host 0.0.0.0] [--device 0]\n"
          "            [--max-batch 8] [--act-dim 23] [--replan 16] [--act-mean v,..] [--act-std v,..]\n"
          "            [--delta-mask 1,0,..] [--noise-seed 0] [--cameras head,left_wrist,right_wrist]\n"
          "            [--siglip-layers N --gemma-layers N --num-steps N (with --random-weights)] [--selftest]\n");
}

}  // namespace

int main(int argc, char** argv) {
  Options o;
  pi05_default_config(&o.cfg);
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) {
        usage();
        exit(2);
      }
      return argv[++i];
    };
    if (a == "--selftest") return selftest();
    if (a == "--weights") o.weights = val();
    else if (a == "--random-weights") o.random_seed = std::stol(val());
    else if (a == "--port") o.port = std::stoi(val());
    else if (a == "--host") o.host = val();
    else if (a == "--device") o.device = std::stoi(val());
    else if (a == "--max-batch") o.max_batch = std::stoi(val());
    else if (a == "--act-dim") o.act_dim = std::stoi(val());
    else if (a == "--replan") o.replan = std::stoi(val());
    else if (a == "--act-mean") o.mean = parse_list<float>(val());
    else if (a == "--act-std") o.stdv = parse_list<float>(val());
    else if (a == "--delta-mask") o.delta = parse_list<uint8_t>(val());
    else if (a == "--noise-seed") o.noise_seed = std::stoull(val());
    else if (a == "--cameras") o.cameras = split(val());
    else if (a == "--siglip-layers") o.cfg.siglip_layers = std::stoi(val());
    else if (a == "--gemma-layers") o.cfg.gemma_layers = o.cfg.expert_layers = std::stoi(val());
    else if (a == "--num-steps") o.cfg.num_steps = std::stoi(val());
    else {
      usage();
      return 2;
    }
  }
  if ((o.weights.empty()) == (o.random_seed < 0)) {
    usage();
    return 2;
  }
  if ((!o.mean.empty() && (int)o.mean.size() != o.act_dim) || o.mean.size() != o.stdv.size() ||
      (!o.delta.empty() && (int)o.delta.size() != o.act_dim)) {
    fprintf(stderr, "pi05_server: --act-mean/--act-std/--delta-mask need act_dim values each\n");
    return 2;
  }
  char err[512] = {0};
  pi05_engine* e = nullptr;
  if (!o.weights.empty()) {
    if (pi05_read_weights_config(o.weights.c_str(), &o.cfg) != PI05_OK) {
      fprintf(stderr, "pi05_server: cannot read %s\n", o.weights.c_str());
      return 1;
    }
    e = pi05_create(&o.cfg, o.device, o.max_batch, err, sizeof err);
    if (e && pi05_load_weights(e, o.weights.c_str()) != PI05_OK) {
      fprintf(stderr, "pi05_server: %s\n", pi05_last_error(e));
      return 1;
    }
  } else {
    e = pi05_create(&o.cfg, o.device, o.max_batch, err, sizeof err);
    if (e && pi05_init_random_weights(e, (uint64_t)o.random_seed) != PI05_OK) {
      fprintf(stderr, "pi05_server: %s\n", pi05_last_error(e));
      return 1;
    }
  }
  if (!e) {
    fprintf(stderr, "pi05_server: %s\n", err);
    return 1;
  }
  if ((int)o.cameras.size() != o.cfg.n_cameras) {
    fprintf(stderr, "pi05_server: %zu camera keys for a %d-camera model\n", o.cameras.size(), o.cfg.n_cameras);
    return 2;
  }
  pi05_act_config ac = {o.act_dim, o.replan, o.mean.empty() ? nullptr : o.mean.data(),
                        o.stdv.empty() ? nullptr : o.stdv.data(), o.delta.empty() ? nullptr : o.delta.data(),
                        o.noise_seed};
  if (pi05_set_act_config(e, &ac) != PI05_OK) {
    fprintf(stderr, "pi05_server: %s\n", pi05_last_error(e));
    return 2;
  }
  signal(SIGPIPE, SIG_IGN);
  const int ls = socket(AF_INET, SOCK_STREAM, 0);
  int one = 1;
  setsockopt(ls, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in addr = {};
  addr.sin_family = AF_INET;
  addr.sin_port = htons((uint16_t)o.port);
  if (inet_pton(AF_INET, o.host.c_str(), &addr.sin_addr) != 1 || bind(ls, (sockaddr*)&addr, sizeof addr) != 0 ||
      listen(ls, 16) != 0) {
    perror("pi05_server: bind/listen");
    return 1;
  }
  printf("pi05_server listening on %s:%d\n", o.host.c_str(), o.port);
  fflush(stdout);
  for (;;) {
    const int fd = accept(ls, nullptr, nullptr);
    if (fd < 0) continue;
    std::thread([fd, e, &o]() {
      serve(fd, e, o);
      close(fd);
    }).detach();
  }
}
