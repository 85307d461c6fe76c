! Drop-in replacement of module matmul_3p5bit_groq (matmul_3p5bit_dynamic.f90) over
! libq35.so: same module name, procedure names, argument order, intents and value
! attributes.  Each procedure takes an optional stat= argument (0 = success, else a
! libq35 status); without it a failure stops the program with libq35's message, as the
! reference's own error paths stop (matmul_cublas.f90:116-117).
! Link: gfortran -c q35_status.f90 matmul_3p5bit_groq.f90 && ... -L<pkg> -lq35 -Wl,-rpath,<pkg>
! C callers keep the reference's bind(C) symbol matmul_3p5bit_awq, which libq35 exports.
module matmul_3p5bit_groq
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    implicit none
    private
    public :: matmul_3p5bit_awq, dequantize_output_3p5bit

    interface
        integer(c_int) function q35_matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, C, M, N, K) &
                bind(C, name="q35_matmul_3p5bit_awq")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(M, K)
            integer(c_int8_t), intent(in) :: W_Q(K/2, N)
            real(c_float), intent(in) :: W_scales(N), W_offsets(N)
            integer(c_int32_t), intent(inout) :: C(M, N)
        end function q35_matmul_3p5bit_awq

        integer(c_int) function q35_dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N) &
                bind(C, name="q35_dequantize_output_3p5bit")
            import :: c_int, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N
            integer(c_int32_t), intent(in) :: C(M, N)
            real(c_float), intent(in) :: W_scales(N), W_offsets(N)
            real(c_float), intent(inout) :: Out(M, N)
        end function q35_dequantize_output_3p5bit
    end interface

contains

    ! matmul_3p5bit_dynamic.f90:28-65
    subroutine matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, C, M, N, K, stat)
        integer(int32), intent(in), value :: M, N, K
        integer(int8), intent(in) :: A(M, K)
        integer(int8), intent(in) :: W_Q(K/2, N)
        real(real32), intent(in) :: W_scales(N), W_offsets(N)
        integer(int32), intent(out) :: C(M, N)
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, C, M, N, K), &
                       "matmul_3p5bit_awq", stat)
    end subroutine matmul_3p5bit_awq

    ! matmul_3p5bit_dynamic.f90:69-82
    subroutine dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N, stat)
        integer(int32), intent(in), value :: M, N
        integer(int32), intent(in) :: C(M, N)
        real(real32), intent(in) :: W_scales(N), W_offsets(N)
        real(real32), intent(out) :: Out(M, N)
        integer, intent(out), optional :: stat
        call q35_check(q35_dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N), &
                       "dequantize_output_3p5bit", stat)
    end subroutine dequantize_output_3p5bit

end module matmul_3p5bit_groq
