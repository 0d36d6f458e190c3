/* host_xfer.h - host <-> device copies of pageable host buffers for the
 * backend vtable (cuda_backend.c). */
#ifndef SAM3CU_HOST_XFER_H
#define SAM3CU_HOST_XFER_H

#include <stddef.h>

struct hxfer;

struct hxfer *hxfer_create(void);
void hxfer_destroy(struct hxfer *x);
/* dev <- host, n bytes, on `stream`; returns when `host` may be reused */
int hxfer_h2d(struct hxfer *x, void *dev, const void *host, size_t n, void *stream);
/* host <- dev after the work queued on `stream`; returns when host holds it */
int hxfer_d2h(struct hxfer *x, void *host, const void *dev, size_t n, void *stream);

#endif
