/* Exercise of the minimpi library on host buffers (no GPU needed): ring
 * Sendrecv of a message larger than the channel, Isend/Irecv with Testall
 * polling, Reduce(MAX) / Allreduce(SUM), Bcast, Comm_split_type, Wtime.
 * Prints "ok <rank>" on success; exits non-zero on the first mismatch. */
#include <mpi.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define N (3 * 1024 * 1024 + 17) /* floats: 12 MiB, crosses several fragments */

static int fail(int rank, const char* what, long i) {
  fprintf(stderr, "rank %d: %s mismatch at %ld\n", rank, what, i);
  MPI_Abort(MPI_COMM_WORLD, 3);
  return 3;
}

int main(int argc, char** argv) {
  int provided = -1, rank, size;
  if (MPI_Init_thread(&argc, &argv, MPI_THREAD_FUNNELED, &provided) != MPI_SUCCESS) return 1;
  if (provided < MPI_THREAD_FUNNELED) return 2;
  MPI_Comm_rank(MPI_COMM_WORLD, &rank);
  MPI_Comm_size(MPI_COMM_WORLD, &size);
  const int right = (rank + 1) % size, left = (rank - 1 + size) % size;
  float* a = (float*)malloc(sizeof(float) * N);
  float* b = (float*)malloc(sizeof(float) * N);
  for (long i = 0; i < N; ++i) a[i] = rank * 1000.0f + (float)(i % 4096);
  /* ring of size-1 steps, like the reference's comm loops */
  for (int step = 0; step < size - 1; ++step) {
    MPI_Status st;
    MPI_Sendrecv(a, N, MPI_FLOAT, right, step, b, N, MPI_FLOAT, left, step, MPI_COMM_WORLD, &st);
    const int src = (rank - step - 1 + 2 * size) % size;
    if (st.MPI_SOURCE != left || st.MPI_TAG != step) return fail(rank, "status", step);
    for (long i = 0; i < N; i += 997)
      if (b[i] != src * 1000.0f + (float)(i % 4096)) return fail(rank, "sendrecv", i);
    float* t = a; a = b; b = t;
  }
  /* non-blocking pair with Testall polling */
  MPI_Request reqs[2];
  MPI_Irecv(b, 1000, MPI_FLOAT, left, 77, MPI_COMM_WORLD, &reqs[0]);
  for (int i = 0; i < 1000; ++i) a[i] = rank + i * 0.5f;
  MPI_Isend(a, 1000, MPI_FLOAT, right, 77, MPI_COMM_WORLD, &reqs[1]);
  int done = 0;
  while (!done) MPI_Testall(2, reqs, &done, MPI_STATUSES_IGNORE);
  for (int i = 0; i < 1000; ++i)
    if (b[i] != left + i * 0.5f) return fail(rank, "isend/irecv", i);
  /* reductions and broadcast */
  double v[5] = {rank, -rank, 2.0 * rank, 1.0, rank == 1 ? 99.0 : 0.0}, mx[5];
  MPI_Reduce(v, mx, 5, MPI_DOUBLE, MPI_MAX, 0, MPI_COMM_WORLD);
  if (rank == 0 && (mx[0] != size - 1 || mx[1] != 0 || mx[2] != 2.0 * (size - 1) || mx[4] != (size > 1 ? 99.0 : 0.0)))
    return fail(rank, "reduce", 0);
  int one = 1, total = 0;
  MPI_Allreduce(&one, &total, 1, MPI_INT, MPI_SUM, MPI_COMM_WORLD);
  if (total != size) return fail(rank, "allreduce", total);
  unsigned char id[128];
  for (int i = 0; i < 128; ++i) id[i] = rank == 0 ? (unsigned char)(i * 7) : 0;
  MPI_Bcast(id, (int)sizeof(id), MPI_BYTE, 0, MPI_COMM_WORLD);
  for (int i = 0; i < 128; ++i)
    if (id[i] != (unsigned char)(i * 7)) return fail(rank, "bcast", i);
  MPI_Comm local;
  int lr = -1, ls = -1;
  MPI_Comm_split_type(MPI_COMM_WORLD, MPI_COMM_TYPE_SHARED, 0, MPI_INFO_NULL, &local);
  MPI_Comm_rank(local, &lr);
  MPI_Comm_size(local, &ls);
  MPI_Comm_free(&local);
  if (lr != rank || ls != size) return fail(rank, "split_type", lr);
  const double t0 = MPI_Wtime();
  MPI_Barrier(MPI_COMM_WORLD);
  if (MPI_Wtime() < t0) return fail(rank, "wtime", 0);
  if (argc > 1 && strcmp(argv[1], "abort") == 0 && rank == size - 1) MPI_Abort(MPI_COMM_WORLD, 7);
  if (argc > 1 && strcmp(argv[1], "abort") == 0) MPI_Barrier(MPI_COMM_WORLD); /* never completes */
  printf("ok %d\n", rank);
  free(a);
  free(b);
  MPI_Finalize();
  return 0;
}
