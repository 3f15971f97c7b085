/*
 * LD_PRELOAD bandwidth shaper for TCP traffic (e.g. NCCL forced onto its socket transport).
 *
 * Environment (same variables as the reference's shaper, infra/socket_shaper.c there):
 *   ZERO_SOCKET_SHAPER_BW_GBPS      link rate in gigabits/s; unset or <= 0 disables shaping
 *   ZERO_SOCKET_SHAPER_LATENCY_MS   extra delay added to every shaped send
 *   ZERO_SOCKET_SHAPER_BURST_BYTES  token-bucket depth (default 262144)
 *   ZERO_SOCKET_SHAPER_SHARED_NAME  when set, every process using this name draws from one bucket
 *                                   kept in POSIX shared memory (one emulated link for all ranks)
 *   ZERO_SOCKET_SHAPER_STATS_DIR    when set, each process writes socket_shaper_<pid>.json at exit
 *
 * Interposed: send, sendto, sendmsg, sendmmsg, write, writev.  Only IPv4/IPv6 sockets are shaped;
 * files, pipes and Unix sockets pass straight through.  Shaping is a token bucket: a send of n
 * bytes takes n tokens; when the bucket goes negative the caller sleeps for the debt / rate.
 * The shared bucket is protected by a process-shared robust mutex, so a process that dies while
 * holding it does not wedge the others (the next locker marks the state consistent).
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/uio.h>
#include <time.h>
#include <unistd.h>

typedef ssize_t (*send_fn)(int, const void *, size_t, int);
typedef ssize_t (*sendto_fn)(int, const void *, size_t, int, const struct sockaddr *, socklen_t);
typedef ssize_t (*sendmsg_fn)(int, const struct msghdr *, int);
typedef int (*sendmmsg_fn)(int, struct mmsghdr *, unsigned int, int);
typedef ssize_t (*write_fn)(int, const void *, size_t);
typedef ssize_t (*writev_fn)(int, const struct iovec *, int);

struct bucket {
  atomic_int state; /* 0 = fresh, 1 = initialising, 2 = ready */
  pthread_mutex_t mutex;
  double tokens;       /* bytes currently available (may be negative: debt) */
  uint64_t last_ns;    /* last refill time */
};

static struct {
  int enabled;
  double bytes_per_ns;
  double burst;
  uint64_t latency_ns;
  struct bucket *bucket;
  struct bucket private_bucket;
  int shared;
  char stats_dir[512];
  atomic_ullong calls;
  atomic_ullong bytes;
  atomic_ullong sleep_ns;
  send_fn real_send;
  sendto_fn real_sendto;
  sendmsg_fn real_sendmsg;
  sendmmsg_fn real_sendmmsg;
  write_fn real_write;
  writev_fn real_writev;
} g;

static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static uint64_t now_ns(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

static void sleep_ns(uint64_t ns) {
  struct timespec ts = {(time_t)(ns / 1000000000ull), (long)(ns % 1000000000ull)};
  while (nanosleep(&ts, &ts) != 0 && errno == EINTR) {
  }
}

static double env_double(const char *name, double fallback) {
  const char *v = getenv(name);
  if (v == NULL || *v == '\0') return fallback;
  char *end = NULL;
  double d = strtod(v, &end);
  return end == v ? fallback : d;
}

static void bucket_setup(struct bucket *b) {
  pthread_mutexattr_t attr;
  pthread_mutexattr_init(&attr);
  pthread_mutexattr_setpshared(&attr, PTHREAD_PROCESS_SHARED);
  pthread_mutexattr_setrobust(&attr, PTHREAD_MUTEX_ROBUST);
  pthread_mutex_init(&b->mutex, &attr);
  pthread_mutexattr_destroy(&attr);
  b->tokens = g.burst;
  b->last_ns = now_ns();
}

static struct bucket *open_shared_bucket(const char *name) {
  char path[300];
  snprintf(path, sizeof(path), "/%s", name[0] == '/' ? name + 1 : name);
  int fd = shm_open(path, O_CREAT | O_RDWR, 0600);
  if (fd < 0) return NULL;
  if (ftruncate(fd, sizeof(struct bucket)) != 0) {
    close(fd);
    return NULL;
  }
  void *mem = mmap(NULL, sizeof(struct bucket), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (mem == MAP_FAILED) return NULL;
  struct bucket *b = (struct bucket *)mem;
  int expected = 0;
  if (atomic_compare_exchange_strong(&b->state, &expected, 1)) {
    bucket_setup(b);
    atomic_store(&b->state, 2);
  } else {
    while (atomic_load(&b->state) != 2) sleep_ns(100000);
  }
  return b;
}

static void write_stats(void) {
  if (!g.enabled || g.stats_dir[0] == '\0') return;
  char path[700];
  snprintf(path, sizeof(path), "%s/socket_shaper_%d.json", g.stats_dir, (int)getpid());
  FILE *f = fopen(path, "w");
  if (f == NULL) return;
  fprintf(f,
          "{\"pid\": %d, \"bandwidth_gbps\": %.6f, \"burst_bytes\": %.0f, \"latency_ms\": %.3f, \"shared\": %s, "
          "\"total_shaped_calls\": %llu, \"total_shaped_bytes\": %llu, \"total_bandwidth_sleep_s\": %.6f}\n",
          (int)getpid(), g.bytes_per_ns * 8.0, g.burst, (double)g.latency_ns / 1e6, g.shared ? "true" : "false",
          (unsigned long long)atomic_load(&g.calls), (unsigned long long)atomic_load(&g.bytes),
          (double)atomic_load(&g.sleep_ns) / 1e9);
  fclose(f);
}

static void init_once(void) {
  g.real_send = (send_fn)dlsym(RTLD_NEXT, "send");
  g.real_sendto = (sendto_fn)dlsym(RTLD_NEXT, "sendto");
  g.real_sendmsg = (sendmsg_fn)dlsym(RTLD_NEXT, "sendmsg");
  g.real_sendmmsg = (sendmmsg_fn)dlsym(RTLD_NEXT, "sendmmsg");
  g.real_write = (write_fn)dlsym(RTLD_NEXT, "write");
  g.real_writev = (writev_fn)dlsym(RTLD_NEXT, "writev");
  const double gbps = env_double("ZERO_SOCKET_SHAPER_BW_GBPS", 0.0);
  g.enabled = gbps > 0.0;
  if (!g.enabled) return;
  g.bytes_per_ns = gbps / 8.0; /* gigabits/s -> bytes/ns */
  g.burst = env_double("ZERO_SOCKET_SHAPER_BURST_BYTES", 262144.0);
  if (g.burst < 1.0) g.burst = 1.0;
  g.latency_ns = (uint64_t)(env_double("ZERO_SOCKET_SHAPER_LATENCY_MS", 0.0) * 1e6);
  const char *stats = getenv("ZERO_SOCKET_SHAPER_STATS_DIR");
  if (stats != NULL) snprintf(g.stats_dir, sizeof(g.stats_dir), "%s", stats);
  const char *shared = getenv("ZERO_SOCKET_SHAPER_SHARED_NAME");
  g.bucket = NULL;
  if (shared != NULL && *shared != '\0') {
    g.bucket = open_shared_bucket(shared);
    g.shared = g.bucket != NULL;
  }
  if (g.bucket == NULL) {
    bucket_setup(&g.private_bucket);
    g.bucket = &g.private_bucket;
  }
  atexit(write_stats);
}

static void ensure_init(void) { pthread_once(&g_once, init_once); }

static int is_inet_socket(int fd) {
  struct sockaddr_storage addr;
  socklen_t len = sizeof(addr);
  if (getsockname(fd, (struct sockaddr *)&addr, &len) != 0) return 0;
  return addr.ss_family == AF_INET || addr.ss_family == AF_INET6;
}

static void lock_bucket(struct bucket *b) {
  if (pthread_mutex_lock(&b->mutex) == EOWNERDEAD) pthread_mutex_consistent(&b->mutex);
}

/* Take `bytes` tokens; sleep off any debt outside the lock. */
static void shape(int fd, size_t bytes) {
  if (!g.enabled || bytes == 0 || !is_inet_socket(fd)) return;
  struct bucket *b = g.bucket;
  lock_bucket(b);
  const uint64_t now = now_ns();
  const double refill = (double)(now - b->last_ns) * g.bytes_per_ns;
  b->last_ns = now;
  b->tokens += refill;
  if (b->tokens > g.burst) b->tokens = g.burst;
  b->tokens -= (double)bytes;
  const double debt = b->tokens < 0.0 ? -b->tokens : 0.0;
  pthread_mutex_unlock(&b->mutex);
  const uint64_t wait = (uint64_t)(debt / g.bytes_per_ns) + g.latency_ns;
  atomic_fetch_add(&g.calls, 1);
  atomic_fetch_add(&g.bytes, (unsigned long long)bytes);
  if (wait > 0) {
    atomic_fetch_add(&g.sleep_ns, wait);
    sleep_ns(wait);
  }
}

static size_t iov_bytes(const struct iovec *iov, size_t n) {
  size_t total = 0;
  for (size_t i = 0; i < n; ++i) total += iov[i].iov_len;
  return total;
}

ssize_t send(int fd, const void *buf, size_t len, int flags) {
  ensure_init();
  shape(fd, len);
  return g.real_send(fd, buf, len, flags);
}

ssize_t sendto(int fd, const void *buf, size_t len, int flags, const struct sockaddr *dst, socklen_t dlen) {
  ensure_init();
  shape(fd, len);
  return g.real_sendto(fd, buf, len, flags, dst, dlen);
}

ssize_t sendmsg(int fd, const struct msghdr *msg, int flags) {
  ensure_init();
  if (msg != NULL) shape(fd, iov_bytes(msg->msg_iov, msg->msg_iovlen));
  return g.real_sendmsg(fd, msg, flags);
}

int sendmmsg(int fd, struct mmsghdr *vec, unsigned int vlen, int flags) {
  ensure_init();
  size_t total = 0;
  for (unsigned int i = 0; vec != NULL && i < vlen; ++i) total += iov_bytes(vec[i].msg_hdr.msg_iov, vec[i].msg_hdr.msg_iovlen);
  shape(fd, total);
  return g.real_sendmmsg(fd, vec, vlen, flags);
}

ssize_t write(int fd, const void *buf, size_t len) {
  ensure_init();
  if (fd > 2) shape(fd, len);
  return g.real_write(fd, buf, len);
}

ssize_t writev(int fd, const struct iovec *iov, int n) {
  ensure_init();
  if (fd > 2 && n > 0) shape(fd, iov_bytes(iov, (size_t)n));
  return g.real_writev(fd, iov, n);
}
