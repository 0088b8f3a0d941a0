/* Host-side failures of the library: the message becomes the one
 * cwen_cuda_last_error() returns (one message per process, shared with the
 * engine), so that callers read host and device failures the same way. */
#ifndef CWEN_HOST_ERR_H
#define CWEN_HOST_ERR_H
#include <stdarg.h>
#include <stdio.h>

/* Defined with the engine's error state (csrc/capi.cu). */
void cwen_host_set_error(const char *msg);

/* Record the formatted message and return rc. */
static inline int host_fail(int rc, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  cwen_host_set_error(buf);
  return rc;
}
#endif
